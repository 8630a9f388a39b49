// GQA decode attention with fused rotary embedding and KV-cache append.
//
// Grid (B, n_kv_heads, S): CTA (b, g, s) serves the G = n_heads / n_kv_heads
// query heads that share KV head g (HF repeat_kv grouping: query head h uses KV
// head h / G) over keys [s * ATT_SPLIT_KEYS, (s + 1) * ATT_SPLIT_KEYS) of
// sequence b.  Only the ceil(L / ATT_SPLIT_KEYS) CTAs whose range holds keys do
// work (L = positions[b] + 1); the rest return at once.
//   1. RoPE (HF half-split convention, bf16 op-by-op like transformers'
//      apply_rotary_pos_emb on bf16 tensors):
//        out[i]    = bf16(bf16(x[i] * cos_i)    + bf16(-x[i+64] * sin_i))
//        out[i+64] = bf16(bf16(x[i+64] * cos_i) + bf16( x[i]    * sin_i))
//      on the G query heads and the new key; the CTA whose range holds the new
//      position writes the rotated key and the value to row positions[b].
//   2. Each warp streams 16-key tiles of K and V (4 KB each, rows contiguous in
//      the cache) with bulk copies into a double buffer of its own and keeps an
//      online softmax: scores q . k_t * scale in fp32 (lane = key x half of the
//      head dimension), running max / sum, and the weighted sum of v_t (lane =
//      4 dimensions).  The tile holding the new position takes the rotated key
//      and the value from shared memory, not from the cache row being written.
//   3. The warps' states merge in shared memory.  With one active CTA the
//      result is normalised and written; otherwise each CTA writes its
//      (max, sum, unnormalised accumulator) to the workspace and the last CTA
//      of (b, g) to arrive (a counter in the workspace, reset by that CTA) merges
//      the parts.
#pragma once
#include "common.cuh"

namespace bitnet {

constexpr int ATT_THREADS = 128;
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int ATT_D = 128;
constexpr int ATT_MAX_G = 8;
constexpr int ATT_TILE = 16;                            // keys per warp tile
constexpr int ATT_NBUF = 2;                             // tiles in flight per warp
constexpr int ATT_TILE_BYTES = ATT_TILE * ATT_D * 2;    // K (or V) of one tile
constexpr int ATT_SPLIT_KEYS = 256;                     // keys per CTA
constexpr int ATT_TILES_BYTES = ATT_WARPS * ATT_NBUF * 2 * ATT_TILE_BYTES;

struct AttnParams {
  const uint16_t* qkv;
  int n_heads, n_kv, G;
  const int32_t* positions;
  const uint16_t* rope_cos;
  const uint16_t* rope_sin;
  int rope_len;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int max_len, max_ctx, nsplit;
  float scale;
  int* ws_count;    // [B * n_kv] arrival counters (zero between launches)
  float* ws_part;   // [B * n_kv * nsplit][2G + G * 128]
  uint16_t* out;
};

__host__ __device__ __forceinline__ int att_part_floats(int G) { return 2 * G + G * ATT_D; }
__host__ __device__ __forceinline__ size_t att_smem_bytes(int G) {
  return (size_t)ATT_TILES_BYTES + (size_t)G * ATT_D * 2 + 2 * ATT_D * 2 + ATT_WARPS * ATT_NBUF * 8;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
  }
}

template <int G>
__global__ void __launch_bounds__(ATT_THREADS) gqa_decode_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_att[];
  uint8_t* tiles = smem_att;                                               // [warp][buf][K | V]
  uint16_t* q_s = reinterpret_cast<uint16_t*>(smem_att + ATT_TILES_BYTES);  // [G][128] rotated queries
  uint16_t* knew = q_s + G * ATT_D;                                        // rotated new key
  uint16_t* vnew = knew + ATT_D;                                           // new value
  uint64_t* bars = reinterpret_cast<uint64_t*>(vnew + ATT_D);             // [warp][buf]
  __shared__ int s_abort, s_last;

  pdl_trigger();  // the next kernel may launch; it waits for this grid before reading
  const int b = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < ATT_WARPS * ATT_NBUF; ++i) mbar_init(&bars[i], 1);
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  const int pos = p.positions[b];
  if (pos < 0 || pos >= p.max_len || pos >= p.rope_len || pos >= p.max_ctx) {
    if (tid == 0 && sp == 0) record_error(DEV_ERR_BOUNDS, 300);
    return;
  }
  const int L = pos + 1;
  const int nparts = (L + ATT_SPLIT_KEYS - 1) / ATT_SPLIT_KEYS;
  if (sp >= nparts) return;
  const int r0 = sp * ATT_SPLIT_KEYS, r1 = min(L, r0 + ATT_SPLIT_KEYS);
  const int ntiles = (r1 - r0 + ATT_TILE - 1) / ATT_TILE;
  const int my_n = ntiles > warp ? (ntiles - warp + ATT_WARPS - 1) / ATT_WARPS : 0;  // tiles of this warp

  const size_t cache_row0 = ((size_t)b * p.n_kv + g) * p.max_len;
  uint16_t* kc = p.k_cache + cache_row0 * ATT_D;
  uint16_t* vc = p.v_cache + cache_row0 * ATT_D;
  auto tile_t0 = [&](int i) { return r0 + (warp + i * ATT_WARPS) * ATT_TILE; };
  auto tile_buf = [&](int i) { return tiles + (size_t)(warp * ATT_NBUF + i % ATT_NBUF) * 2 * ATT_TILE_BYTES; };
  auto tile_bar = [&](int i) { return &bars[warp * ATT_NBUF + i % ATT_NBUF]; };
  // Lane 0 arms the barrier, lanes 0 / 1 copy K / V (a thread's copies run one
  // after another, so the two go out from different lanes).
  auto issue = [&](int i) {
    const int t0 = tile_t0(i), nk = min(ATT_TILE, r1 - t0);
    if (lane == 0) mbar_arrive_expect_tx(tile_bar(i), (uint32_t)(2 * nk * ATT_D * 2));
    __syncwarp();
    if (lane < 2)
      bulk_g2s(tile_buf(i) + lane * ATT_TILE_BYTES, (lane == 0 ? kc : vc) + (size_t)t0 * ATT_D,
               (uint32_t)(nk * ATT_D * 2), tile_bar(i));
  };
  for (int i = 0; i < min(my_n, ATT_NBUF); ++i) issue(i);

  // ---- 1. RoPE on the G query heads and the new key; stage the new value ----
  const int row_elems = (p.n_heads + 2 * p.n_kv) * ATT_D;
  const uint16_t* qkv = p.qkv + (size_t)b * row_elems;
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
      uint16_t* dst = (hh < G) ? q_s + hh * ATT_D : knew;
      dst[i] = f32_to_bf16_bits(o1);
      dst[i + 64] = f32_to_bf16_bits(o2);
    }
  } else {
    const int i = tid - ATT_D / 2;  // 64 threads x 2 values
    reinterpret_cast<uint32_t*>(vnew)[i] =
        reinterpret_cast<const uint32_t*>(qkv + (size_t)(p.n_heads + p.n_kv + g) * ATT_D)[i];
  }
  __syncthreads();
  if (sp == nparts - 1 && tid < 32) {  // append row `pos` (16 B per lane: 16 lanes K, 16 lanes V)
    const int part = tid >> 4, c = tid & 15;
    uint16_t* dst = (part == 0 ? kc : vc) + (size_t)pos * ATT_D;
    const uint16_t* src = part == 0 ? knew : vnew;
    reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
  }

  // ---- 2. scores, online softmax, P.V ----
  float m_run[G], l_run[G], acc[G][4];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    m_run[hh] = -INFINITY;
    l_run[hh] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[hh][j] = 0.f;
  }
  const int key = lane & (ATT_TILE - 1), half = lane >> 4;
  int waited = 0;  // tiles whose copies this warp has seen land
  for (int i = 0; i < my_n; ++i) {
    const int t0 = tile_t0(i), nk = min(ATT_TILE, r1 - t0);
    uint8_t* buf = tile_buf(i);
    if (!__all_sync(0xffffffffu, mbar_wait(tile_bar(i), (uint32_t)((i / ATT_NBUF) & 1), 301))) {
      if (lane == 0) s_abort = 1;
      break;
    }
    waited = i + 1;
    if (pos >= t0 && pos < t0 + nk) {  // the new row: take it from shared memory
      uint32_t* kr = reinterpret_cast<uint32_t*>(buf + (pos - t0) * ATT_D * 2);
      uint32_t* vr = reinterpret_cast<uint32_t*>(buf + ATT_TILE_BYTES + (pos - t0) * ATT_D * 2);
      kr[lane] = reinterpret_cast<const uint32_t*>(knew)[lane];
      kr[lane + 32] = reinterpret_cast<const uint32_t*>(knew)[lane + 32];
      vr[lane] = reinterpret_cast<const uint32_t*>(vnew)[lane];
      vr[lane + 32] = reinterpret_cast<const uint32_t*>(vnew)[lane + 32];
      __syncwarp();
    }
    // scores: lane (key, half) dots 64 dimensions; 16-byte chunks are visited in
    // a key-rotated order so the 8 lanes of a shared-memory phase hit 8
    // different bank groups
    float sc[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) sc[hh] = 0.f;
    if (key < nk) {
      const uint8_t* krow = buf + key * ATT_D * 2 + half * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int ch = (c + key) & 7;
        float kf[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(krow + ch * 16), kf);
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
          float qf[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(q_s + hh * ATT_D + half * 64 + ch * 8), qf);
#pragma unroll
          for (int e = 0; e < 8; ++e) sc[hh] = fmaf(kf[e], qf[e], sc[hh]);
        }
      }
    }
    float pr[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      const float full_dot = sc[hh] + __shfl_xor_sync(0xffffffffu, sc[hh], 16);
      const float s = (key < nk) ? full_dot * p.scale : -INFINITY;
      float mx = s;
#pragma unroll
      for (int o = ATT_TILE / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run[hh], mx);
      const float corr = expf(m_run[hh] - m_new);  // exp(-inf) = 0 on the first tile
      const float e = (key < nk) ? expf(s - m_new) : 0.f;
      float es = e;
#pragma unroll
      for (int o = ATT_TILE / 2; o > 0; o >>= 1) es += __shfl_xor_sync(0xffffffffu, es, o);
      l_run[hh] = l_run[hh] * corr + es;
      m_run[hh] = m_new;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[hh][j] *= corr;
      pr[hh] = e;
    }
    const uint8_t* vb = buf + ATT_TILE_BYTES + lane * 8;
#pragma unroll
    for (int j = 0; j < ATT_TILE; ++j) {
      if (j < nk) {
        const uint2 vv = *reinterpret_cast<const uint2*>(vb + j * ATT_D * 2);
        const float v0 = __uint_as_float(vv.x << 16), v1 = __uint_as_float(vv.x & 0xFFFF0000u);
        const float v2 = __uint_as_float(vv.y << 16), v3 = __uint_as_float(vv.y & 0xFFFF0000u);
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
    // Reuse the buffer: every lane is done reading it (generic proxy) before
    // the bulk copy (async proxy) overwrites it.
    __syncwarp();
    if (i + ATT_NBUF < my_n) {
      fence_proxy_async_smem();
      issue(i + ATT_NBUF);
    }
  }
  // Copies still in flight after an abort land before shared memory is reused.
  for (int i = waited; i < min(my_n, waited + ATT_NBUF); ++i) mbar_wait(tile_bar(i), (uint32_t)((i / ATT_NBUF) & 1), 302);
  __syncthreads();
  if (s_abort) return;

  // ---- 3. merge the warp states (tile buffers are free now) ----
  float* sm_m = reinterpret_cast<float*>(tiles);      // [warp][G]
  float* sm_l = sm_m + ATT_WARPS * G;                 // [warp][G]
  float* sm_acc = sm_l + ATT_WARPS * G;               // [warp][G][128]
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    if (lane == 0) {
      sm_m[warp * G + hh] = m_run[hh];
      sm_l[warp * G + hh] = l_run[hh];
    }
    *reinterpret_cast<float4*>(sm_acc + (warp * G + hh) * ATT_D + lane * 4) =
        make_float4(acc[hh][0], acc[hh][1], acc[hh][2], acc[hh][3]);
  }
  __syncthreads();
  uint16_t* out_b = p.out + (size_t)b * p.n_heads * ATT_D + (size_t)g * G * ATT_D;
  const size_t pf = (size_t)att_part_floats(G);
  float* part_base = p.ws_part + ((size_t)b * p.n_kv + g) * p.nsplit * pf;
  for (int idx = tid; idx < G * ATT_D; idx += ATT_THREADS) {
    const int hh = idx / ATT_D, d = idx % ATT_D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, sm_m[w * G + hh]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) {
      const float f = (sm_l[w * G + hh] > 0.f) ? expf(sm_m[w * G + hh] - M) : 0.f;
      num = fmaf(sm_acc[(w * G + hh) * ATT_D + d], f, num);
      den = fmaf(sm_l[w * G + hh], f, den);
    }
    if (nparts == 1) {
      out_b[idx] = f32_to_bf16_bits(num / den);
    } else {
      float* part = part_base + sp * pf;
      if (d == 0) {
        part[hh] = M;
        part[G + hh] = den;
      }
      part[2 * G + idx] = num;
    }
  }
  if (nparts == 1) return;

  // ---- 4. the last CTA of (b, g) merges the parts ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int* cnt = p.ws_count + (size_t)b * p.n_kv + g;
    const int old = atomicAdd(cnt, 1);
    s_last = (old == nparts - 1);
    if (s_last) atomicExch(cnt, 0);  // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < G * ATT_D; idx += ATT_THREADS) {
    const int hh = idx / ATT_D;
    float M = -INFINITY;
    for (int s = 0; s < nparts; ++s) M = fmaxf(M, __ldcg(part_base + s * pf + hh));
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nparts; ++s) {
      const float* part = part_base + s * pf;
      const float ls = __ldcg(part + G + hh);
      const float f = (ls > 0.f) ? expf(__ldcg(part + hh) - M) : 0.f;
      num = fmaf(__ldcg(part + 2 * G + idx), f, num);
      den = fmaf(ls, f, den);
    }
    out_b[idx] = f32_to_bf16_bits(num / den);
  }
}

}  // namespace bitnet
