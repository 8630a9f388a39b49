// lm_head (tied embedding, bf16) with fused greedy argmax.
//
// logits[b, v] = bf16(sum_k h[b, k] * W[v, k])   (fp32 accumulation, one bf16
// rounding, as a bf16 nn.Linear); token[b] = argmax_v logits[b, v] with the
// smallest index winning ties (torch.argmax).  Stage 1 computes one 128-row
// vocabulary tile per CTA and writes the tile's per-token (max, index) pair to
// the workspace; stage 2 reduces the pairs of all tiles per token, writes the
// token id and advances the sequence's decode position.
#pragma once
#include "common.cuh"
#include "pack.cuh"

namespace bitnet {

struct ArgPair {
  float v;
  int i;
};
__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

constexpr int LMH_THREADS = 128;
constexpr int LMH_TOK = 32;  // tokens per pass

// grid.x = Vpad / 128.  dynamic smem: h as [K/8][B] uint4 (B <= 32).
__global__ void __launch_bounds__(LMH_THREADS)
lm_head_simt_kernel(const uint16_t* __restrict__ h, int B, int K, const uint4* __restrict__ w_tiled, int V,
                    int KC8, ArgPair* __restrict__ part, uint16_t* __restrict__ logits_out) {
  extern __shared__ __align__(16) uint4 sh[];
  __shared__ float red_v[LMH_THREADS / 32][LMH_TOK];
  __shared__ int red_i[LMH_THREADS / 32][LMH_TOK];
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vt = blockIdx.x;
  const int v = vt * 128 + tid;
  // stage h: sh[c * B + b] = h[b, 8c .. 8c+7]
  for (int i = tid; i < KC8 * B; i += LMH_THREADS) {
    const int c = i / B, b = i % B;
    uint16_t e[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = c * 8 + j;
      e[j] = (k < K) ? h[(size_t)b * K + k] : (uint16_t)0;
    }
    sh[i] = make_uint4((uint32_t)e[0] | ((uint32_t)e[1] << 16), (uint32_t)e[2] | ((uint32_t)e[3] << 16),
                       (uint32_t)e[4] | ((uint32_t)e[5] << 16), (uint32_t)e[6] | ((uint32_t)e[7] << 16));
  }
  __syncthreads();

  float acc[LMH_TOK];
#pragma unroll
  for (int b = 0; b < LMH_TOK; ++b) acc[b] = 0.f;
  const uint4* wrow = w_tiled + lm_layout_offset16(v, 0, KC8);
  for (int c = 0; c < KC8; ++c) {
    const uint4 wv = wrow[(size_t)c * 128];
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    float wf[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wf[2 * j] = bf16_bits_to_f32((uint16_t)(ww[j] & 0xFFFF));
      wf[2 * j + 1] = bf16_bits_to_f32((uint16_t)(ww[j] >> 16));
    }
#pragma unroll
    for (int b = 0; b < LMH_TOK; ++b) {
      if (b < B) {
        const uint4 hv = sh[c * B + b];
        const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
        float a = acc[b];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a = fmaf(wf[2 * j], bf16_bits_to_f32((uint16_t)(hw[j] & 0xFFFF)), a);
          a = fmaf(wf[2 * j + 1], bf16_bits_to_f32((uint16_t)(hw[j] >> 16)), a);
        }
        acc[b] = a;
      }
    }
  }

  // per-token argmax over the tile's 128 rows
#pragma unroll
  for (int b = 0; b < LMH_TOK; ++b) {
    if (b >= B) break;
    const float lg = round_bf16(acc[b]);
    if (logits_out != nullptr && v < V) logits_out[(size_t)b * V + v] = f32_to_bf16_bits(lg);
    float bv = (v < V) ? lg : -INFINITY;
    int bi = (v < V) ? v : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (arg_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      red_v[warp][b] = bv;
      red_i[warp][b] = bi;
    }
  }
  __syncthreads();
  pdl_trigger();
  if (tid < B) {
    float bv = red_v[0][tid];
    int bi = red_i[0][tid];
    for (int w = 1; w < LMH_THREADS / 32; ++w)
      if (arg_better(red_v[w][tid], red_i[w][tid], bv, bi)) {
        bv = red_v[w][tid];
        bi = red_i[w][tid];
      }
    part[(size_t)vt * B + tid] = ArgPair{bv, bi};
  }
}

// grid = B, block = 256.
__global__ void __launch_bounds__(256)
argmax_reduce_kernel(const ArgPair* __restrict__ part, int ntiles, int B, int32_t* __restrict__ out_ids,
                     int32_t* __restrict__ positions) {
  __shared__ float sv[256];
  __shared__ int si[256];
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = tid; t < ntiles; t += 256) {
    const ArgPair a = part[(size_t)t * B + b];
    if (arg_better(a.v, a.i, bv, bi)) {
      bv = a.v;
      bi = a.i;
    }
  }
  sv[tid] = bv;
  si[tid] = bi;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s && arg_better(sv[tid + s], si[tid + s], sv[tid], si[tid])) {
      sv[tid] = sv[tid + s];
      si[tid] = si[tid + s];
    }
    __syncthreads();
  }
  if (tid == 0) {
    out_ids[b] = si[0];
    if (positions != nullptr) positions[b] += 1;
  }
  pdl_trigger();
}

}  // namespace bitnet
