// CUDA-core BitLinear for small token counts (the decode regime below the
// ridge batch).  HBM-bound: each weight byte is read once, unpacked in
// registers to four int8 codes and fed to __dp4a against every token.
//
// CTA = 8 warps.  A CTA owns 32 consecutive weight rows (64 for the RELU2_MUL
// epilogue: one 32-row gate group and its matching 32-row up group); lane l of
// a warp owns row n0 + l, and the warps split K.  Per 64-weight chunk a lane
// issues one 16-byte streaming load, so a warp reads 512 contiguous bytes.
// The quantised activation rows (at most 8) sit in shared memory and are read
// as warp-wide broadcasts.
#pragma once
#include "act_quant.cuh"
#include "common.cuh"
#include "epilogue.cuh"

namespace bitnet {

__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

constexpr int SIMT_THREADS = 256;
constexpr int SIMT_MAX_M = 8;
constexpr int SIMT_REG_CHUNKS = 16;  // 64-wide K chunks a lane holds in registers at once (16 B each)

// Fused mode: the CTA computes the RMSNorm + int8 act-quant of the (at most 8)
// token rows itself, straight into its shared-memory code tile, instead of
// reading codes that a separate act-quant launch wrote.  x == nullptr: off.
struct SimtFuse {
  const uint16_t* x;  // bf16 [M, ldx], rows 16-byte aligned
  int ldx, K;
  const uint16_t* gamma;  // nullable
  float eps;
};

// grid.x = ceil(N / rows_per_cta).  dynamic smem = Kp * 8 (q rows 0..7) + reduction.
template <int EPI, int MT>
__global__ void __launch_bounds__(SIMT_THREADS, 2)
bitlinear_simt_kernel(const int8_t* __restrict__ q, const float* __restrict__ row_scale,
                      const int32_t* __restrict__ row_sum, int M, int Kp, int T, const uint8_t* __restrict__ w,
                      int N, bitnet_segments_dev seg, const uint16_t* residual, uint16_t* y,
                      int32_t* __restrict__ acc_out, const SimtFuse fz) {
  constexpr int RG = (EPI == EPI_RELU2_MUL) ? 2 : 1;  // 32-row groups per CTA
  constexpr int KS = 8 / RG;                          // K splits per row group
  extern __shared__ __align__(16) uint8_t smem_simt[];
  uint8_t* smem = smem_simt;
  uint4* sq = reinterpret_cast<uint4*>(smem);                     // [Kp/16][8 rows] x 16 B
  int* sred = reinterpret_cast<int*>(smem + (size_t)Kp * 8);      // [8 warps][MT][32]
  __shared__ float s_scale[SIMT_MAX_M];  // fused mode: per-token scale and code sum
  __shared__ int s_sum[SIMT_MAX_M];
  __shared__ double s_rd[AQ_THREADS / 32];
  __shared__ float s_rf[AQ_THREADS / 32];
  __shared__ int s_ri[AQ_THREADS / 32];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rg = warp / KS, ks = warp % KS;
  const int n0 = blockIdx.x * (32 * RG);
  const int n = n0 + rg * 32 + lane;
  const int KC = Kp >> 6;
  const int kc_begin = (ks * KC) / KS, kc_end = ((ks + 1) * KC) / KS;

  const uint8_t* wrow = w + wlayout_offset(n, 0, KC);
  const int nch = kc_end - kc_begin;

  // The lane's weight chunks (up to SIMT_REG_CHUNKS at once) are loaded before
  // griddepcontrol.wait: the weights do not come from the previous kernel, so
  // their HBM reads overlap it; only the activation codes wait.
  uint4 wv[SIMT_REG_CHUNKS];
  auto load_w = [&](int b0) {
#pragma unroll
    for (int u = 0; u < SIMT_REG_CHUNKS; ++u)
      wv[u] = (b0 + u < nch) ? ldg_stream16(wrow + (size_t)(kc_begin + b0 + u) * 2048u) : make_uint4(0, 0, 0, 0);
  };
  pdl_trigger();  // the next kernel may launch; it waits for this grid before reading
  load_w(0);
  const bool fused = fz.x != nullptr;
  uint4 gr[AQ_MAXC];
  if (fused) aq_load_gamma(gr, fz.gamma, fz.K, tid);  // gamma does not come from the previous kernel either
  pdl_wait();
  if (fused) {
    // sq is the code layout of a token tile of 8 rows: for each 16-wide K chunk
    // 8 rows x 16 B, i.e. the act-quant layout with T = 8
    const AqScratch sc{s_rd, s_rf, s_ri};
    for (int m = 0; m < M; ++m)
      aq_row_vec<0>(fz.x, M, fz.K, fz.ldx, fz.gamma != nullptr, gr, fz.eps, reinterpret_cast<int8_t*>(sq), s_scale,
                    s_sum, nullptr, 8, Kp, m, sc, tid);
  } else {
    // Stage the tile's q rows 0..MT-1: for each 16-wide K chunk the first rows of
    // its first core matrix (8 rows x 16 B).
    const int C16 = Kp >> 4;
    for (int i = tid; i < C16 * MT; i += SIMT_THREADS) {
      const int c = i / MT, r = i % MT;
      sq[c * 8 + r] = *reinterpret_cast<const uint4*>(q + ((size_t)c * (T >> 3)) * 128u + (size_t)r * 16u);
    }
  }
  __syncthreads();

  int acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0;

  for (int b0 = 0; b0 < nch; b0 += SIMT_REG_CHUNKS) {
    if (b0 > 0) load_w(b0);
    const int kc0 = kc_begin + b0;
#pragma unroll
    for (int u = 0; u < SIMT_REG_CHUNKS; ++u) {
      if (b0 + u >= nch) break;
      const uint32_t xw[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        uint32_t c0, c1, c2, c3;
        unpack16(xw[wi], c0, c1, c2, c3);
        const int c16 = (kc0 + u) * 4 + wi;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < M) {
            const uint4 qv = sq[c16 * 8 + m];
            int a = acc[m];
            a = __dp4a((int)c0, (int)qv.x, a);
            a = __dp4a((int)c1, (int)qv.y, a);
            a = __dp4a((int)c2, (int)qv.z, a);
            a = __dp4a((int)c3, (int)qv.w, a);
            acc[m] = a;
          }
        }
      }
    }
  }

#pragma unroll
  for (int m = 0; m < MT; ++m) sred[(warp * MT + m) * 32 + lane] = acc[m];
  __syncthreads();

  if (EPI == EPI_RELU2_MUL) {
    // pairs p (32) x tokens m: gate row n0 + p, up row n0 + 32 + p
    for (int i = tid; i < 32 * MT; i += SIMT_THREADS) {
      const int p = i & 31, m = i >> 5;
      if (m >= M) continue;
      const int ng = n0 + p, nu = n0 + 32 + p;
      if (nu >= N) continue;
      int ag = 0, au = 0;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        ag += sred[((0 * KS + s) * MT + m) * 32 + p];
        au += sred[((1 * KS + s) * MT + m) * 32 + p];
      }
      const int rsm = fused ? s_sum[m] : row_sum[m];
      ag -= rsm;
      au -= rsm;
      if (acc_out) {
        acc_out[(size_t)m * N + ng] = ag;
        acc_out[(size_t)m * N + nu] = au;
      }
      const float sm = fused ? s_scale[m] : row_scale[m];
      const float g = scaled_bf16(ag, seg.scale[0], sm);
      const float u = scaled_bf16(au, seg.scale[1], sm);
      const int o = (n0 >> 6) * 32 + p;
      y[(size_t)m * (N >> 1) + o] = relu2_mul_bf16(g, u);
    }
  } else {
    for (int i = tid; i < 32 * MT; i += SIMT_THREADS) {
      const int r = i & 31, m = i >> 5;
      if (m >= M) continue;
      const int nn = n0 + r;
      if (nn >= N) continue;
      int a = 0;
#pragma unroll
      for (int s = 0; s < KS; ++s) a += sred[(s * MT + m) * 32 + r];
      a -= fused ? s_sum[m] : row_sum[m];
      if (acc_out) acc_out[(size_t)m * N + nn] = a;
      const float v = scaled_bf16(a, seg_scale_of(seg, nn), fused ? s_scale[m] : row_scale[m]);
      const size_t o = (size_t)m * N + nn;
      if (EPI == EPI_RESIDUAL_ADD)
        y[o] = residual_add_bf16(residual[o], v);
      else
        y[o] = f32_to_bf16_bits(v);
    }
  }
}

}  // namespace bitnet
