// tcgen05 BitLinear: int8 activations x ternary weights on the 5th-generation
// tensor cores, for batches at and above the ridge (decode batch 32, prefill).
//
// Roles of the operands (one CTA = one 128-row weight tile x one token tile):
//   A (M = 128 weight rows, K)  lives in TENSOR MEMORY.  Each of the 128 threads
//       owns one weight row, reads its packed 2-bit row slice from shared memory,
//       unpacks it in registers to int8 codes c = w + 1 in {0,1,2} and writes them
//       with tcgen05.st.  The 4x expansion of the weights therefore never touches
//       shared memory: smem only carries the packed bytes and the activations.
//   B (N = T tokens, K) is the quantised activation tile, moved by a bulk copy
//       straight into the canonical K-major core-matrix layout.
//   D (128 x T, int32) accumulates in tensor memory.
// acc' = sum_k c_k q_k is exact in int32; the epilogue subtracts row_sum[m] to
// recover the ternary accumulator.
//
// Pipeline: packed weights and activations of each 256-wide K stage arrive by
// bulk copy into a ring of `nslot` shared-memory slots (one mbarrier each).  A
// is double-buffered in TMEM (2 x 64 columns); the MMAs of a stage are
// committed to the mbarrier of their A buffer.  The weight copies of the first
// slots are issued before griddepcontrol.wait, so with programmatic dependent
// launch they overlap the tail of the previous kernel.
//
// K split: when the grid's z extent (= cluster size) is > 1, the CTAs of one
// cluster own disjoint K ranges of the same tile, park their partial D in
// shared memory and reduce through distributed shared memory; each CTA of the
// cluster finishes a disjoint set of tokens.  No global scratch is used.
#pragma once
#include "common.cuh"
#include "epilogue.cuh"

namespace bitnet {

constexpr int TC_THREADS = 128;
constexpr int TC_STAGE_CHUNKS = 4;  // 4 x 64 = 256 K positions per stage
constexpr int TC_MAX_SLOTS = 16;
constexpr int TC_CTRL_BYTES = 1024;

struct TcParams {
  const int8_t* q;
  const float* row_scale;
  const int32_t* row_sum;
  int M, Kp, T;  // tokens, padded K, token tile height (multiple of 16, <= 256)
  const uint8_t* w;
  int N, KC;  // output rows, K chunks of 64
  bitnet_segments_dev seg;
  const uint16_t* residual;
  uint16_t* y;
  int32_t* acc_out;
  int nslot;
  int split;
};

__host__ __device__ __forceinline__ int tc_slot_bytes(int T) { return TC_STAGE_CHUNKS * 2048 + TC_STAGE_CHUNKS * 64 * T; }
__host__ __device__ __forceinline__ int tc_tmem_cols(int T) { return (128 + T) <= 256 ? 256 : 512; }

struct TcCtrl {
  uint64_t full[TC_MAX_SLOTS];
  uint64_t mma_done[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) bitlinear_tc_kernel(const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_tc[];
  uint8_t* smem = smem_tc;
  TcCtrl* ctrl = reinterpret_cast<TcCtrl*>(smem);
  uint8_t* ring = smem + TC_CTRL_BYTES;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int nb = blockIdx.x, mt = blockIdx.y, ks = blockIdx.z;
  const int T = p.T, KC = p.KC, nslot = p.nslot, split = p.split;
  const int kc_begin = (ks * KC) / split, kc_end = ((ks + 1) * KC) / split;
  const int nstages = (kc_end - kc_begin + TC_STAGE_CHUNKS - 1) / TC_STAGE_CHUNKS;
  const int slot_bytes = tc_slot_bytes(T);
  const int wslot_bytes = TC_STAGE_CHUNKS * 2048;
  const uint32_t ncols = tc_tmem_cols(T);
  const uint32_t idesc = idesc_i8_s32(128, T);
  volatile int* abort_flag = &ctrl->abort_flag;

  if (tid == 0) {
    for (int s = 0; s < nslot; ++s) mbar_init(&ctrl->full[s], 1);
    mbar_init(&ctrl->mma_done[0], 1);
    mbar_init(&ctrl->mma_done[1], 1);
    ctrl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&ctrl->tmem_base, ncols);
    tmem_relinquish();
  }
  // Announce that this CTA is running; peers wait on it before their first
  // distributed-shared-memory store into this CTA.
  if (split > 1) cluster_arrive_relaxed();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctrl->tmem_base;
  const uint32_t tmem_d = tbase + 128;

  uint64_t policy = 0;
  auto stage_chunks = [&](int s) { return min(TC_STAGE_CHUNKS, kc_end - (kc_begin + s * TC_STAGE_CHUNKS)); };
  auto issue_weights = [&](int s) {
    const int slot = s % nslot, nch = stage_chunks(s);
    const int kc_s = kc_begin + s * TC_STAGE_CHUNKS;
    mbar_arrive_expect_tx(&ctrl->full[slot], (uint32_t)(nch * 2048 + nch * 64 * T));
    bulk_g2s_stream(ring + (size_t)slot * slot_bytes, p.w + ((size_t)nb * KC + kc_s) * 2048u, nch * 2048,
                    &ctrl->full[slot], policy);
  };
  auto issue_acts = [&](int s) {
    const int slot = s % nslot, nch = stage_chunks(s);
    const int kc_s = kc_begin + s * TC_STAGE_CHUNKS;
    bulk_g2s(ring + (size_t)slot * slot_bytes + wslot_bytes, p.q + (size_t)mt * T * p.Kp + (size_t)kc_s * 64 * T,
             nch * 64 * T, &ctrl->full[slot]);
  };

  int issued = 0;  // stages whose copies have been issued (thread 0 only)
  const int prologue = min(nslot, nstages);
  if (tid == 0) {
    policy = l2_policy_evict_first();
    for (int s = 0; s < prologue; ++s) issue_weights(s);
  }
  pdl_wait();
  if (tid == 0) {
    for (int s = 0; s < prologue; ++s) issue_acts(s);
    issued = prologue;
  }

  auto wait_or_abort = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity, site)) {
      *abort_flag = 1;
      return false;
    }
    return true;
  };

  for (int s = 0; s < nstages; ++s) {
    const int slot = s % nslot;
    const int ab = s & 1;
    const int nch = stage_chunks(s);
    bool ok = true;
    if (s >= 2) ok = wait_or_abort(&ctrl->mma_done[ab], ((s >> 1) + 1) & 1, 200);
    if (ok) ok = wait_or_abort(&ctrl->full[slot], (s / nslot) & 1, 201);
    if (ok) {
      const uint8_t* wsm = ring + (size_t)slot * slot_bytes;
      const uint32_t tst = tbase + ((uint32_t)(warp * 32) << 16) + ab * 64;
      for (int c = 0; c < nch; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(wsm + c * 2048 + tid * 16);
        uint32_t o[16];
        unpack16(v.x, o[0], o[1], o[2], o[3]);
        unpack16(v.y, o[4], o[5], o[6], o[7]);
        unpack16(v.z, o[8], o[9], o[10], o[11]);
        unpack16(v.w, o[12], o[13], o[14], o[15]);
        tmem_st16(tst + c * 16, o);
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && !*abort_flag) {
      tc_fence_after();
      const uint32_t a_base = tbase + ab * 64;
      const uint32_t b_base = smem_u32(ring + (size_t)slot * slot_bytes + wslot_bytes);
      for (int kk = 0; kk < 2 * nch; ++kk) {
        const uint64_t bdesc = smem_desc_kmajor(b_base + kk * 32 * T, 16 * T, 128);
        mma_i8_ts(tmem_d, a_base + kk * 8, bdesc, idesc, (s | kk) != 0 ? 1u : 0u);
      }
      tc_commit(&ctrl->mma_done[ab]);
      // Refill the slot of stage s-1 once its MMAs (the previous commit) are done.
      if (s >= 1 && issued < nstages) {
        if (wait_or_abort(&ctrl->mma_done[(s - 1) & 1], ((s - 1) >> 1) & 1, 202)) {
          issue_weights(issued);
          issue_acts(issued);
          ++issued;
        }
      }
    }
  }

  // All MMAs done -> D is final for this CTA.
  if (nstages > 0) wait_or_abort(&ctrl->mma_done[(nstages - 1) & 1], ((nstages - 1) >> 1) & 1, 203);
  tc_fence_after();
  pdl_trigger();

  // Partial D (128 rows x T tokens, int32) -> the owner of each token.
  // Token m belongs to cluster rank (m * split) / T; rank j owns tokens
  // [ceil(j*T/split), ceil((j+1)*T/split)).  Without a split the single CTA owns
  // all tokens and stages them in the (now idle) ring.
  const int cr = (split > 1) ? (int)cluster_ctarank() : 0;
  const int tok_cap = (T + split - 1) / split;  // tokens per owner, upper bound
  const int ldr = tok_cap + 1;                  // odd row stride: conflict-free
  int* recv = reinterpret_cast<int*>(split > 1 ? ring + (size_t)nslot * slot_bytes : ring);
  const uint32_t recv_base = smem_u32(recv);
  if (split > 1) cluster_wait();  // every peer of the cluster has started
  if (!*abort_flag) {
    const uint32_t tld = tmem_d + ((uint32_t)(warp * 32) << 16);
    for (int c = 0; c < T; c += 16) {
      uint32_t v[16];
      tmem_ld16(tld + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = c + j;
        const int owner = (m * split) / T;
        const int mm = m - (owner * T + split - 1) / split;
        const int idx = (cr * 128 + tid) * ldr + mm;
        if (owner == cr)
          recv[idx] = (int)v[j];
        else
          st_shared_cluster_s32(mapa_shared(recv_base + (uint32_t)idx * 4u, (uint32_t)owner), (int)v[j]);
      }
    }
  }
  tc_fence_before();
  if (split > 1)
    cluster_sync();
  else
    __syncthreads();

  const bool aborted = *abort_flag != 0;
  const int m_begin = (cr * T + split - 1) / split, m_end = ((cr + 1) * T + split - 1) / split;
  auto partial = [&](int row, int m) -> int {
    int a = 0;
    for (int j = 0; j < split; ++j) a += recv[(j * 128 + row) * ldr + (m - m_begin)];
    return a;
  };
  const int N = p.N;

  if (!aborted) {
    if (EPI == EPI_RELU2_MUL) {
      const int pr = tid & 63;   // pair within the tile
      const int half = tid >> 6; // two threads share a pair, splitting tokens
      const int g0 = (pr >> 5) * 64 + (pr & 31);  // gate row in tile; up row = g0 + 32
      const int ng = nb * 128 + g0, nu = ng + 32;
      for (int m = m_begin + half; m < m_end; m += 2) {
        const int mg = mt * T + m;
        if (mg >= p.M || nu >= N) continue;
        const int rs = p.row_sum[mg];
        const int ag = partial(g0, m) - rs;
        const int au = partial(g0 + 32, m) - rs;
        if (p.acc_out) {
          p.acc_out[(size_t)mg * N + ng] = ag;
          p.acc_out[(size_t)mg * N + nu] = au;
        }
        const float sm = p.row_scale[mg];
        const float g = scaled_bf16(ag, p.seg.scale[0], sm);
        const float u = scaled_bf16(au, p.seg.scale[1], sm);
        p.y[(size_t)mg * (N >> 1) + nb * 64 + (g0 >> 6) * 32 + (g0 & 31)] = relu2_mul_bf16(g, u);
      }
    } else {
      const int row = tid;
      const int n = nb * 128 + row;
      const float wsc = seg_scale_of(p.seg, n);
      for (int m = m_begin; m < m_end; ++m) {
        const int mg = mt * T + m;
        if (mg >= p.M || n >= N) continue;
        const int a = partial(row, m) - p.row_sum[mg];
        if (p.acc_out) p.acc_out[(size_t)mg * N + n] = a;
        const float v = scaled_bf16(a, wsc, p.row_scale[mg]);
        const size_t o = (size_t)mg * N + n;
        if (EPI == EPI_RESIDUAL_ADD)
          p.y[o] = residual_add_bf16(p.residual[o], v);
        else
          p.y[o] = f32_to_bf16_bits(v);
      }
    }
  }

  if (tid == 0 && aborted) {
    // Let every copy this CTA may still have in flight land before its shared
    // memory is released: the most recent fill of each slot.
    for (int s = max(0, issued - nslot); s < issued; ++s) mbar_wait(&ctrl->full[s % nslot], (s / nslot) & 1, 204);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, ncols);
  }
}

}  // namespace bitnet
