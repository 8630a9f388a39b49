// GQA decode attention with fused rotary embedding and KV-cache append.
//
// One CTA per (sequence b, KV head g); it serves the G = n_heads / n_kv_heads
// query heads that share KV head g (HF repeat_kv grouping: query head h uses
// KV head h / G).
//   1. RoPE (HF half-split convention, bf16 op-by-op like
//      transformers' apply_rotary_pos_emb on bf16 tensors):
//        out[i]    = bf16(bf16(x[i] * cos_i)      + bf16(-x[i+64] * sin_i))
//        out[i+64] = bf16(bf16(x[i+64] * cos_i)   + bf16( x[i]    * sin_i))
//      applied to the G query heads and the new key; the rotated key and the
//      value are written to row positions[b] of the caches.
//   2. softmax(q . k_t * scale) over t = 0 .. positions[b] (inclusive) and the
//      weighted sum of v_t, in fp32, with an online softmax per warp (warps own
//      interleaved blocks of 32 keys; a lane scores one key of the block) and a
//      final merge of the warp states in shared memory.
#pragma once
#include "common.cuh"

namespace bitnet {

constexpr int ATT_THREADS = 256;
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int ATT_D = 128;
constexpr int ATT_MAX_G = 8;

struct AttnParams {
  const uint16_t* qkv;
  int n_heads, n_kv, G;
  const int32_t* positions;
  const uint16_t* rope_cos;
  const uint16_t* rope_sin;
  int rope_len;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int max_len;
  float scale;
  uint16_t* out;
};

template <int G>
__global__ void __launch_bounds__(ATT_THREADS) gqa_decode_kernel(const AttnParams p) {
  __shared__ float sq[G][ATT_D];
  __shared__ float sm_m[ATT_WARPS][G];
  __shared__ float sm_l[ATT_WARPS][G];
  __shared__ float sm_acc[ATT_WARPS][G][ATT_D];

  pdl_trigger();  // the next kernel may launch; it waits for this grid before reading
  pdl_wait();
  const int b = blockIdx.x, g = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = p.positions[b];
  if (pos < 0 || pos >= p.max_len || pos >= p.rope_len) {
    if (tid == 0) record_error(DEV_ERR_BOUNDS, 300);
    return;
  }
  const int row_elems = (p.n_heads + 2 * p.n_kv) * ATT_D;
  const uint16_t* qkv = p.qkv + (size_t)b * row_elems;
  const size_t cache_row0 = ((size_t)b * p.n_kv + g) * p.max_len;
  uint16_t* kc = p.k_cache + cache_row0 * ATT_D;
  uint16_t* vc = p.v_cache + cache_row0 * ATT_D;

  // ---- 1. RoPE on the G query heads and the new key; append K and V ----
  if (tid < ATT_D / 2) {
    const int i = tid;
    const float c = bf16_bits_to_f32(p.rope_cos[(size_t)pos * (ATT_D / 2) + i]);
    const float s = bf16_bits_to_f32(p.rope_sin[(size_t)pos * (ATT_D / 2) + i]);
#pragma unroll
    for (int hh = 0; hh <= G; ++hh) {
      const uint16_t* src = (hh < G) ? qkv + (size_t)(g * G + hh) * ATT_D : qkv + (size_t)(p.n_heads + g) * ATT_D;
      const float x1 = bf16_bits_to_f32(src[i]);
      const float x2 = bf16_bits_to_f32(src[i + 64]);
      const float o1 = round_bf16(__fadd_rn(round_bf16(__fmul_rn(x1, c)), round_bf16(__fmul_rn(-x2, s))));
      const float o2 = round_bf16(__fadd_rn(round_bf16(__fmul_rn(x2, c)), round_bf16(__fmul_rn(x1, s))));
      if (hh < G) {
        sq[hh][i] = o1;
        sq[hh][i + 64] = o2;
      } else {
        kc[(size_t)pos * ATT_D + i] = f32_to_bf16_bits(o1);
        kc[(size_t)pos * ATT_D + i + 64] = f32_to_bf16_bits(o2);
      }
    }
  } else if (tid < ATT_D / 2 + ATT_D) {
    const int i = tid - ATT_D / 2;
    vc[(size_t)pos * ATT_D + i] = qkv[(size_t)(p.n_heads + p.n_kv + g) * ATT_D + i];
  }
  __syncthreads();

  // ---- 2. scores, online softmax, P.V ----
  const int L = pos + 1;
  float m_run[G], l_run[G], acc[G][4];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    m_run[hh] = -INFINITY;
    l_run[hh] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[hh][j] = 0.f;
  }

  for (int j0 = warp * 32; j0 < L; j0 += ATT_WARPS * 32) {
    const int t = j0 + lane;
    float sc[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) sc[hh] = 0.f;
    if (t < L) {
      const uint4* krow = reinterpret_cast<const uint4*>(kc + (size_t)t * ATT_D);
#pragma unroll 4
      for (int c8 = 0; c8 < ATT_D / 8; ++c8) {
        const uint4 kv = krow[c8];
        const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float k0 = bf16_bits_to_f32((uint16_t)(kw[e] & 0xFFFF));
          const float k1 = bf16_bits_to_f32((uint16_t)(kw[e] >> 16));
          const int d = c8 * 8 + 2 * e;
#pragma unroll
          for (int hh = 0; hh < G; ++hh) sc[hh] = fmaf(k0, sq[hh][d], fmaf(k1, sq[hh][d + 1], sc[hh]));
        }
      }
    }
    float pr[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      const float s = (t < L) ? sc[hh] * p.scale : -INFINITY;
      float mx = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run[hh], mx);
      const float corr = expf(m_run[hh] - m_new);  // exp(-inf) = 0 on the first block
      const float e = (t < L) ? expf(s - m_new) : 0.f;
      float es = e;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) es += __shfl_xor_sync(0xffffffffu, es, o);
      l_run[hh] = l_run[hh] * corr + es;
      m_run[hh] = m_new;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[hh][j] *= corr;
      pr[hh] = e;
    }
    const int nkeys = min(32, L - j0);
    for (int j = 0; j < nkeys; ++j) {
      const uint2 vv = *reinterpret_cast<const uint2*>(vc + (size_t)(j0 + j) * ATT_D + lane * 4);
      const float v0 = bf16_bits_to_f32((uint16_t)(vv.x & 0xFFFF)), v1 = bf16_bits_to_f32((uint16_t)(vv.x >> 16));
      const float v2 = bf16_bits_to_f32((uint16_t)(vv.y & 0xFFFF)), v3 = bf16_bits_to_f32((uint16_t)(vv.y >> 16));
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        const float pj = __shfl_sync(0xffffffffu, pr[hh], j);
        acc[hh][0] = fmaf(pj, v0, acc[hh][0]);
        acc[hh][1] = fmaf(pj, v1, acc[hh][1]);
        acc[hh][2] = fmaf(pj, v2, acc[hh][2]);
        acc[hh][3] = fmaf(pj, v3, acc[hh][3]);
      }
    }
  }

  // ---- 3. merge the warp states ----
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    if (lane == 0) {
      sm_m[warp][hh] = m_run[hh];
      sm_l[warp][hh] = l_run[hh];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) sm_acc[warp][hh][lane * 4 + j] = acc[hh][j];
  }
  __syncthreads();
  for (int i = tid; i < G * ATT_D; i += ATT_THREADS) {
    const int hh = i / ATT_D, d = i % ATT_D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, sm_m[w][hh]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) {
      const float f = (sm_l[w][hh] > 0.f) ? expf(sm_m[w][hh] - M) : 0.f;
      num = fmaf(sm_acc[w][hh][d], f, num);
      den = fmaf(sm_l[w][hh], f, den);
    }
    p.out[(size_t)b * p.n_heads * ATT_D + (size_t)(g * G + hh) * ATT_D + d] = f32_to_bf16_bits(num / den);
  }
}

}  // namespace bitnet
