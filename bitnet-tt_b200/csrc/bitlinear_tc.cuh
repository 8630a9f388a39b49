// tcgen05 BitLinear: int8 activations x ternary weights on the 5th-generation
// tensor cores, for batches at and above the ridge (decode batch 32, prefill).
//
// Roles of the operands (one CTA = one 128-row weight tile x one token tile):
//   A (M = 128 weight rows, K) lives in TENSOR MEMORY.  Unpacker warps read
//       the packed 2-bit rows from shared memory, expand them in registers to
//       int8 codes c = w + 1 in {0,1,2} and write them with tcgen05.st, so the
//       4x expansion of the weights never touches shared memory.
//   B (N = T tokens, K) is the quantised activation tile, moved by bulk copy
//       straight into the canonical K-major core-matrix layout.
//   D (128 x T, int32) accumulates in tensor memory.
// acc' = sum_k c_k q_k is exact in int32; the epilogue subtracts row_sum[m].
//
// Warp roles (384 threads):
//   warps 0-7   unpackers: warp w owns TMEM lane quarter w % 4 and half of the
//               four 64-wide K chunks of a stage; after tcgen05.wait::st each
//               warp arrives on the A buffer's `a_full` barrier.  A is a ring
//               of up to 8 buffers (all of TMEM not taken by D): an MMA
//               completes ~0.5-0.8 us after issue, so the unpackers must be
//               able to run that far ahead;
//   warps 8-10  MMA issuers: lane 0 of issuer i issues the stage's K steps
//               kk = i, i+NACC, ... into its own accumulator D_i (more than
//               one issuing thread: one thread alone issues at most one MMA
//               per ~36 ns, too slow at small N); each issuer commits to the
//               A buffer's `a_empty`, the slot's `slot_free` and, at the end,
//               `d_final`;
//   warp 11     producer: bulk copies of packed weights and activations into a
//               ring of shared-memory slots (weights of the first slots before
//               griddepcontrol.wait, so they overlap the previous kernel), the
//               tile's per-token scales / row sums into shared memory, refills.
// Epilogue without a K split: all 12 warps read D (tcgen05.ld; warp w reads
// lane quarter w % 4), finish each value to its bf16 result and stage the tile
// token-major in the idle ring; then they write whole output rows with 16-byte
// stores (residual read in batches ahead of the stores).  With a K split (grid
// z = cluster size > 1) the unpacker warps sum D_0..D_{NACC-1} into shared
// memory, every CTA pushes each token's partials into the CTA of the cluster
// that owns the token through distributed shared memory, and each owner
// finishes its tokens.  No global scratch is used.
#pragma once
#include "common.cuh"
#include "epilogue.cuh"

namespace bitnet {

constexpr int TC_UNPACK_WARPS = 8;
constexpr int TC_ISSUE_WARP0 = 8;
constexpr int TC_PRODUCER_WARP = 11;
// 12 warps: two CTAs then spread evenly over the SM's four sub-partitions (a
// 13-warp CTA puts a fourth warp on one of them, and the register budget of a
// sub-partition then admits only one CTA per SM)
constexpr int TC_THREADS = 12 * 32;
constexpr int TC_EPI_THREADS = TC_UNPACK_WARPS * 32;
constexpr int TC_STAGE_CHUNKS = 4;  // 4 x 64 = 256 K positions per stage (prefill; TcParams::sc)
constexpr int TC_MAX_STAGE_CHUNKS = 8;  // decode stages: up to 8 x 64 = 512 K positions
constexpr int TC_MAX_SLOTS = 16;
constexpr int TC_MAX_NBUF = 8;      // A buffers in TMEM (64 columns each)
constexpr int TC_TMEM_COLS = 512;       // one CTA per SM; 256 when two CTAs share an SM
constexpr int TC_CTRL_BYTES = 5120;
constexpr int TC_ST_LD = 136;  // bf16 row stride of the staged output tile (272 B: rows stay 16-byte aligned)

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
  int nbuf;  // A buffers in TMEM
  int tmem_cols;  // 512 (one CTA per SM) or 256 (two)
  int sc;         // K chunks of 64 per stage: 4 (prefill), up to TC_MAX_STAGE_CHUNKS at decode
};

__host__ __device__ __forceinline__ int tc_slot_bytes(int T, int sc = TC_STAGE_CHUNKS) { return sc * 2048 + sc * 64 * T; }
// K split: rank j of the cluster owns tokens [j * tok_cap, (j + 1) * tok_cap);
// one CTA's partial sums for one owner are tok_cap tokens x 128 rows int32,
// token-major, so a warp (32 consecutive rows) writes and reads 128
// contiguous bytes per token.
__host__ __device__ __forceinline__ int tc_tok_cap(int T, int split) { return (T + split - 1) / split; }
__host__ __device__ __forceinline__ int tc_part_bytes(int T, int split) { return 128 * tc_tok_cap(T, split) * 4; }
// tokens owned by cluster rank r
__host__ __device__ __forceinline__ int tc_tok_own(int T, int split, int r) {
  const int cap = tc_tok_cap(T, split), b = r * cap, e = b + cap < T ? b + cap : T;
  return e > b ? e - b : 0;
}
__host__ __device__ __forceinline__ int tc_nacc(int T) { return T <= 32 ? 3 : (T <= 64 ? 2 : 1); }
// A buffers of sc chunks (16 * sc TMEM columns each) beside the accumulators
__host__ __device__ __forceinline__ int tc_nbuf(int T, int cols = TC_TMEM_COLS, int sc = TC_STAGE_CHUNKS) {
  const int nb = (cols - tc_nacc(T) * T) / (16 * sc);
  return nb > TC_MAX_NBUF ? TC_MAX_NBUF : nb;
}

struct TcCtrl {
  uint64_t w_full[TC_MAX_SLOTS];  // the slot's packed weights have landed
  uint64_t x_full[TC_MAX_SLOTS];  // the slot's activation codes have landed
  uint64_t slot_free[TC_MAX_SLOTS];
  uint64_t a_full[TC_MAX_NBUF];
  uint64_t a_empty[TC_MAX_NBUF];
  uint64_t d_final;
  uint64_t recv_full;  // split > 1: the peers' partials for this CTA's tokens have landed
  uint32_t tmem_base;
  int abort_flag;
  // 16-byte aligned: the epilogue reads them as int4 / float4
  alignas(16) float scale[256];  // row_scale of the tile's tokens
  alignas(16) int rsum[256];     // row_sum of the tile's tokens
  alignas(16) float fac0[256];   // w_scale / row_scale per token (gate scale for RELU2_MUL)
  alignas(16) float fac1[256];   // up scale / row_scale per token (RELU2_MUL)
};

static_assert(sizeof(TcCtrl) <= TC_CTRL_BYTES, "control block");
static_assert(offsetof(TcCtrl, rsum) % 16 == 0 && offsetof(TcCtrl, fac0) % 16 == 0 &&
                  offsetof(TcCtrl, fac1) % 16 == 0,
              "vector reads of the per-token arrays");

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 2) bitlinear_tc_kernel(const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_tc[];
  TcCtrl* ctrl = reinterpret_cast<TcCtrl*>(smem_tc);
  uint8_t* ring = smem_tc + TC_CTRL_BYTES;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = blockIdx.x, mt = blockIdx.y, ks = blockIdx.z;
  const int T = p.T, KC = p.KC, nslot = p.nslot, split = p.split, NB = p.nbuf, SC = p.sc;
  const int NACC = tc_nacc(T);
  const int kc_begin = (ks * KC) / split, kc_end = ((ks + 1) * KC) / split;
  const int nstages = (kc_end - kc_begin + SC - 1) / SC;
  // Every CTA of a launch reads the same activation block.  Starting each CTA
  // at a different K stage spreads those reads over the L2 instead of having
  // all SMs hit the same lines at once; the integer sum is order-independent.
  const int rot = nstages > 0 ? (int)((blockIdx.x + blockIdx.y * 7u) % (unsigned)nstages) : 0;
  const int slot_bytes = tc_slot_bytes(T, SC);
  const int wslot_bytes = SC * 2048;
  const int acols = 16 * SC;  // TMEM columns of one A buffer
  const uint32_t ncols = (uint32_t)p.tmem_cols;
  volatile int* abort_flag = &ctrl->abort_flag;

  if (tid == 0) {
    for (int s = 0; s < nslot; ++s) {
      mbar_init(&ctrl->w_full[s], 1);
      mbar_init(&ctrl->x_full[s], 1);
      mbar_init(&ctrl->slot_free[s], NACC);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&ctrl->a_full[b], TC_UNPACK_WARPS);
      mbar_init(&ctrl->a_empty[b], NACC);
    }
    mbar_init(&ctrl->d_final, NACC);
    mbar_init(&ctrl->recv_full, 1);
    // every peer sends 128 rows x 4 bytes for each token this CTA owns
    if (split > 1)
      mbar_arrive_expect_tx(&ctrl->recv_full,
                            (uint32_t)((split - 1) * 128 * 4 * tc_tok_own(T, split, (int)cluster_ctarank())));
    ctrl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&ctrl->tmem_base, ncols);
    tmem_relinquish();
  }
  // Announce that this CTA runs; peers wait on it before their first
  // distributed-shared-memory store into this CTA.
  if (split > 1) cluster_arrive_relaxed();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The next kernel may launch now: its CTAs can start their own weight
  // prefetch while this one runs; it waits for this grid before reading it.
  pdl_trigger();
  // Every thread waits for the whole cluster here, at the start (the CTAs of
  // a cluster are co-scheduled), so the barrier's latency overlaps the weight
  // prefetch instead of delaying the partial-sum exchange after the MMAs.
  if (split > 1) cluster_wait();
  const uint32_t tbase = ctrl->tmem_base;
  const uint32_t tmem_d = tbase + NB * acols;  // D_i at tmem_d + i * T

  // logical stage s -> K chunks [kc0(s), kc0(s) + stage_chunks(s))
  auto kc0 = [&](int s) {
    int g = s + rot;
    if (g >= nstages) g -= nstages;
    return kc_begin + g * SC;
  };
  auto stage_chunks = [&](int s) { return min(SC, kc_end - kc0(s)); };
  auto wait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity, site)) {
      *abort_flag = 1;
      return false;
    }
    return true;
  };
  // on-chip hand-offs (A buffer full / empty): poll without suspending
  auto wait_spin = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait_spin(bar, parity, site)) {
      *abort_flag = 1;
      return false;
    }
    return true;
  };

  if (warp == TC_PRODUCER_WARP) {
    // ------------------------------ producer ------------------------------
    // A thread's bulk copies complete one after another (~0.3 us each), so the
    // prologue spreads them over the lanes: lane s issues slot s.  Each lane
    // only ever waits on barriers armed by other warps.
    const int pre = min(nslot, nstages);
    int issued = 0;
    if (lane < pre) {
      const int s = lane;
      const int nch = stage_chunks(s), kc_s = kc0(s);
      mbar_arrive_expect_tx(&ctrl->w_full[s], (uint32_t)(nch * 2048));
      bulk_g2s_stream(ring + (size_t)s * slot_bytes, p.w + ((size_t)nb * KC + kc_s) * 2048u, nch * 2048,
                      &ctrl->w_full[s], l2_policy_evict_first());
    }
    pdl_wait();
    if (lane < pre) {
      const int s = lane;
      const int nch = stage_chunks(s), kc_s = kc0(s);
      mbar_arrive_expect_tx(&ctrl->x_full[s], (uint32_t)(nch * 64 * T));
      bulk_g2s(ring + (size_t)s * slot_bytes + wslot_bytes, p.q + (size_t)mt * T * p.Kp + (size_t)kc_s * 64 * T,
               nch * 64 * T, &ctrl->x_full[s]);
    }
    // Per-token scale factors (one IEEE division per token, done here while
    // the MMAs run rather than after them): fac0 = w_scale / row_scale (the gate
    // scale for RELU2_MUL), fac1 = up scale / row_scale.  fac0 assumes the
    // tile's rows share one segment; the epilogue divides per element when
    // they do not.
    const float sc0 = (EPI == EPI_RELU2_MUL) ? p.seg.scale[0] : seg_scale_of(p.seg, nb * 128);
    for (int i = lane; i < T; i += 32) {
      const int mg = mt * T + i;
      const float s_i = p.row_scale[mg];
      ctrl->scale[i] = s_i;
      ctrl->rsum[i] = p.row_sum[mg];
      ctrl->fac0[i] = __fdiv_rn(sc0, s_i);
      if (EPI == EPI_RELU2_MUL) ctrl->fac1[i] = __fdiv_rn(p.seg.scale[1], s_i);
    }
    // Refills (only when the K range has more stages than the ring has slots).
    // Lane 0 waits for the slot; the warp stays converged, and a large
    // activation block is split over XPARTS lanes: one thread's bulk copies
    // complete one after another, several threads' copies overlap.
    issued = pre;
    {
      const uint64_t policy = l2_policy_evict_first();
      for (int s = pre; s < nstages; ++s) {
        const int slot = s % nslot;
        // the slot's previous stage (s - nslot) is fully consumed once its MMAs are done
        bool ok = true;
        if (lane == 0) ok = wait(&ctrl->slot_free[slot], ((s / nslot) + 1) & 1, 200);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        const int nch = stage_chunks(s), kc_s = kc0(s);
        const uint32_t xbytes = (uint32_t)(nch * 64 * T);
        const int xparts = xbytes >= 32768u ? 4 : 1;  // xbytes is a multiple of 1024
        if (lane == 0) {
          mbar_arrive_expect_tx(&ctrl->w_full[slot], (uint32_t)(nch * 2048));
          bulk_g2s_stream(ring + (size_t)slot * slot_bytes, p.w + ((size_t)nb * KC + kc_s) * 2048u, nch * 2048,
                          &ctrl->w_full[slot], policy);
          // armed with the whole block before any part is issued
          mbar_arrive_expect_tx(&ctrl->x_full[slot], xbytes);
        }
        __syncwarp();
        if (lane < xparts) {
          const uint32_t part = xbytes / (uint32_t)xparts;
          bulk_g2s(ring + (size_t)slot * slot_bytes + wslot_bytes + lane * part,
                   p.q + (size_t)mt * T * p.Kp + (size_t)kc_s * 64 * T + lane * part, part, &ctrl->x_full[slot]);
        }
        issued = s + 1;
      }
    }
    if (lane == 0) {
      if (*abort_flag) {
        for (int s = max(0, issued - nslot); s < issued; ++s) {
          mbar_wait(&ctrl->w_full[s % nslot], (s / nslot) & 1, 204);
          mbar_wait(&ctrl->x_full[s % nslot], (s / nslot) & 1, 204);
        }
      }
    }
    __syncwarp();
  } else if (warp >= TC_ISSUE_WARP0) {
    // ------------------------------ MMA issuers ------------------------------
    const int iss = warp - TC_ISSUE_WARP0;
    if (lane == 0 && iss < NACC) {
      const uint32_t idesc = idesc_i8_s32(128, T);
      const uint32_t d = tmem_d + iss * T;
      bool first = true;
      for (int s = 0; s < nstages; ++s) {
        const int slot = s % nslot, b = s % NB;
        if (!wait_spin(&ctrl->a_full[b], (s / NB) & 1, 201)) break;
        if (!wait_spin(&ctrl->x_full[slot], (s / nslot) & 1, 207)) break;
        tc_fence_after();
        const uint32_t a_base = tbase + b * acols;
        const uint32_t b_base = smem_u32(ring + (size_t)slot * slot_bytes + wslot_bytes);
        const int ksteps = 2 * stage_chunks(s);
        for (int kk = iss; kk < ksteps; kk += NACC) {
          const uint64_t bdesc = smem_desc_kmajor(b_base + kk * 32 * T, 16 * T, 128);
          mma_i8_ts(d, a_base + kk * 8, bdesc, idesc, first ? 0u : 1u);
          first = false;
        }
        // A tcgen05.commit holds its issuing thread for about a microsecond
        // (measured on B200: a commit every 8 MMAs turns 43 ns per MMA into
        // 166 ns), so an A buffer or ring slot is released only when a later
        // stage of this CTA reuses it; every wait on a_empty / slot_free is
        // for exactly those stages.
        if (s + NB < nstages) tc_commit(&ctrl->a_empty[b]);
        if (s + nslot < nstages) tc_commit(&ctrl->slot_free[slot]);
      }
      tc_commit(&ctrl->d_final);
    }
    __syncwarp();
  } else {
    // ------------------------------ unpackers ------------------------------
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    for (int s = 0; s < nstages; ++s) {
      const int slot = s % nslot, b = s % NB;
      bool ok = true;
      if (s >= NB) ok = wait_spin(&ctrl->a_empty[b], ((s / NB) + 1) & 1, 202);
      // weights only: the unpack does not wait for the activations (those come
      // after griddepcontrol.wait), so the first stages unpack while the
      // previous kernel still runs
      if (ok) ok = wait(&ctrl->w_full[slot], (s / nslot) & 1, 203);
      if (ok) {
        const uint8_t* wsm = ring + (size_t)slot * slot_bytes;
        const uint32_t tst = tbase + ((uint32_t)(quarter * 32) << 16) + b * acols;
        const int nch = stage_chunks(s);
        for (int c = half; c < nch; c += 2) {
          const uint4 v = *reinterpret_cast<const uint4*>(wsm + c * 2048 + row * 16);
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctrl->a_full[b]);
      if (!ok) break;
    }
  }

  // ------------------------------ epilogue ------------------------------
  // Everybody waits for the last MMA of every issuer.
  if (nstages > 0) wait(&ctrl->d_final, 0, 205);
  tc_fence_after();
  __syncthreads();  // scale, row-sum and factor staging by the producer is visible too
  pdl_wait();       // (already satisfied) orders this thread's reads of residual after the predecessor

  // Per-token scale factors, one IEEE division per token instead of one per
  // output.  Valid when the tile's rows share one segment (always true for the
  // fused QKV, whose segment ends are multiples of 128); otherwise the output
  // loop divides per element.
  const int N = p.N;
  const int row_lo = nb * 128, row_hi = min(N, row_lo + 128) - 1;
  const bool seg_uniform = (EPI == EPI_RELU2_MUL) || seg_scale_of(p.seg, row_lo) == seg_scale_of(p.seg, row_hi);
  const int used_acc = min(NACC, 2 * (kc_end - kc_begin));
  const bool small_acc = KC <= 256;  // K <= 16384: |acc| < 2^22, float(acc) by i2f_exact

  if (split == 1) {
    // Whole-K tile: no exchange.  Phase 1: the unpacker warps read D (thread =
    // weight row, 16 tokens per tcgen05.ld), finish each value to its bf16 result
    // and stage it token-major in the (now idle) ring.  Phase 2: all 12 warps
    // write whole output rows with 16-byte stores; the residual is read in
    // batches of 4 vectors per thread before any of their stores, so the loads
    // overlap (y and residual may be the same buffer, which keeps the compiler
    // from moving a load above an earlier store).
    uint16_t* st = reinterpret_cast<uint16_t*>(ring);  // [T][TC_ST_LD] bf16
    if (!*abort_flag) {
      // all 12 warps: warp w reads TMEM lane quarter w % 4 (the rows it may
      // access) and every third 16-token chunk
      const int quarter = warp & 3, third = warp >> 2;
      const int r = quarter * 32 + lane;  // TMEM lane = row of the weight tile
      const int n = nb * 128 + r;
      const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
      // RELU2_MUL rows: 0-31 gates of pairs 0-31, 32-63 their ups, 64-95 gates
      // of pairs 32-63, 96-127 their ups; staged as [gates 0-63 | ups 0-63]
      const bool up = (EPI == EPI_RELU2_MUL) && ((r >> 5) & 1);
      const int col = (EPI == EPI_RELU2_MUL) ? (up ? 64 : 0) + (r & 31) + (r >> 6) * 32 : r;
      const float* fac = up ? ctrl->fac1 : ctrl->fac0;
      const float wsc = seg_scale_of(p.seg, n);
      const bool fast = EPI == EPI_RELU2_MUL || seg_uniform;
      for (int c = third * 16; c < T; c += 48) {
        uint32_t sum[16];
        tmem_ld16(tmem_d + lanes + c, sum);
        tmem_wait_ld();
        for (int a = 1; a < used_acc; ++a) {
          uint32_t v[16];
          tmem_ld16(tmem_d + lanes + a * T + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) sum[j] += v[j];
        }
        int acc[16];
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const int4 rs = *reinterpret_cast<const int4*>(&ctrl->rsum[c + 4 * j4]);
          const float4 f4 = *reinterpret_cast<const float4*>(&fac[c + 4 * j4]);
          const int rsv[4] = {rs.x, rs.y, rs.z, rs.w};
          const float fv[4] = {f4.x, f4.y, f4.z, f4.w};
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 4 * j4 + e, m = c + j;
            acc[j] = (int)sum[j] - rsv[e];
            v[e] = fast ? __fmul_rn(i2f_exact(acc[j], small_acc), fv[e]) : scaled_bf16(acc[j], wsc, ctrl->scale[m]);
          }
          // bf16 of two tokens per conversion (rounding a bf16 value again changes nothing)
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int m = c + 4 * j4 + e;
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[e], v[e + 1]);
            const uint32_t bits = *reinterpret_cast<const uint32_t*>(&b2);
            st[m * TC_ST_LD + col] = (uint16_t)(bits & 0xFFFFu);
            st[(m + 1) * TC_ST_LD + col] = (uint16_t)(bits >> 16);
          }
        }
        if (p.acc_out != nullptr && n < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int mg = mt * T + c + j;
            if (mg < p.M) p.acc_out[(size_t)mg * N + n] = acc[j];
          }
        }
      }
    }
    __syncthreads();
    if (!*abort_flag) {
      constexpr int NCOL = (EPI == EPI_RELU2_MUL) ? 64 : 128;  // outputs of one token in this tile
      constexpr int CH = NCOL / 8;
      const int Nout = (EPI == EPI_RELU2_MUL) ? (N >> 1) : N;
      const int col0 = nb * NCOL;
      const int ncols = min(NCOL, Nout - col0);
      const int mvalid = min(T, p.M - mt * T);
      const bool vec = ((Nout & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0) &&
                       (EPI != EPI_RESIDUAL_ADD || (reinterpret_cast<uintptr_t>(p.residual) & 15) == 0);
      const int items = mvalid * CH;
      constexpr int BATCH = 4;
      for (int i0 = tid; i0 < items; i0 += BATCH * TC_THREADS) {
        uint4 res[BATCH];
        if (EPI == EPI_RESIDUAL_ADD) {
#pragma unroll
          for (int u = 0; u < BATCH; ++u) {
            const int it = i0 + u * TC_THREADS;
            res[u] = make_uint4(0, 0, 0, 0);
            if (it < items) {
              const int m = it / CH, c0 = (it % CH) * 8;
              const size_t o = (size_t)(mt * T + m) * Nout + col0 + c0;
              if (vec && c0 + 8 <= ncols) {
                res[u] = *reinterpret_cast<const uint4*>(p.residual + o);
              } else {
                uint16_t* rs = reinterpret_cast<uint16_t*>(&res[u]);
                for (int e = 0; e < 8 && c0 + e < ncols; ++e) rs[e] = p.residual[o + e];
              }
            }
          }
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const int it = i0 + u * TC_THREADS;
          if (it >= items) break;
          const int m = it / CH, c0 = (it % CH) * 8;
          if (c0 >= ncols) continue;
          const size_t o = (size_t)(mt * T + m) * Nout + col0 + c0;
          const uint16_t* sv = st + m * TC_ST_LD + c0;
          uint4 o4;
          if (EPI == EPI_RELU2_MUL) {
            const uint4 g4 = *reinterpret_cast<const uint4*>(sv);
            const uint4 u4 = *reinterpret_cast<const uint4*>(sv + 64);
            o4 = make_uint4(relu2_mul_bf2(g4.x, u4.x), relu2_mul_bf2(g4.y, u4.y), relu2_mul_bf2(g4.z, u4.z),
                            relu2_mul_bf2(g4.w, u4.w));
          } else {
            const uint4 v4 = *reinterpret_cast<const uint4*>(sv);
            o4 = (EPI == EPI_RESIDUAL_ADD)
                     ? make_uint4(residual_add_bf2(res[u].x, v4.x), residual_add_bf2(res[u].y, v4.y),
                                  residual_add_bf2(res[u].z, v4.z), residual_add_bf2(res[u].w, v4.w))
                     : v4;
          }
          if (vec && c0 + 8 <= ncols) {
            *reinterpret_cast<uint4*>(p.y + o) = o4;
          } else {
            const uint16_t* out = reinterpret_cast<const uint16_t*>(&o4);
            for (int e = 0; e < 8 && c0 + e < ncols; ++e) p.y[o + e] = out[e];
          }
        }
      }
    }
  } else {

  // Partial D -> the owner of each token.  Rank j of the cluster owns tokens
  // [j * tok_cap, min(T, (j + 1) * tok_cap)) and holds one receive slot per
  // source rank (tok_cap tokens x 128 rows, token-major).  Each thread sends
  // its row's partials straight from registers: st.async into the owner's
  // slot, counted on the owner's recv_full barrier, or a plain store for its
  // own share.  A warp's store of one token covers 128 contiguous bytes.
  const int cr = (int)cluster_ctarank();
  const int tok_cap = tc_tok_cap(T, split);
  const int slot_ints = 128 * tok_cap;  // ints per receive slot
  int* recv = reinterpret_cast<int*>(ring + (size_t)nslot * slot_bytes);
  if (warp < TC_UNPACK_WARPS && !*abort_flag) {
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    int* own = recv + (size_t)cr * slot_ints + row;  // this rank's slot, at every owner
    const uint32_t own_s = smem_u32(own), bar_s = smem_u32(&ctrl->recv_full);
    for (int c = half * 16; c < T; c += 32) {
      // every accumulator's chunk in flight at once, one wait
      uint32_t sum[16], v1[16], v2[16];
      tmem_ld16(tmem_d + lanes + c, sum);
      if (used_acc > 1) tmem_ld16(tmem_d + lanes + T + c, v1);
      if (used_acc > 2) tmem_ld16(tmem_d + lanes + 2 * T + c, v2);
      tmem_wait_ld();
      if (used_acc > 1) {
#pragma unroll
        for (int j = 0; j < 16; ++j) sum[j] += v1[j];
      }
      if (used_acc > 2) {
#pragma unroll
        for (int j = 0; j < 16; ++j) sum[j] += v2[j];
      }
      int owner = c / tok_cap;  // one division per 16 tokens
      int obeg = owner * tok_cap;
      uint32_t dst = mapa_shared(own_s, (uint32_t)owner), dbar = mapa_shared(bar_s, (uint32_t)owner);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = c + j;  // < T: T is a multiple of 16
        if (m >= obeg + tok_cap) {
          ++owner;
          obeg += tok_cap;
          dst = mapa_shared(own_s, (uint32_t)owner);
          dbar = mapa_shared(bar_s, (uint32_t)owner);
        }
        if (owner == cr)
          own[(m - obeg) * 128] = (int)sum[j];
        else
          st_async_s32(dst + (uint32_t)(m - obeg) * 512u, (int)sum[j], dbar);
      }
    }
  }
  tc_fence_before();
  __syncthreads();  // this CTA's own share is visible to its epilogue threads
  const int m_begin = cr * tok_cap, m_end = min(T, m_begin + tok_cap);
  // Residual-add owners read their first batch of residual values now, so the
  // L2 round trip overlaps the wait for the peers' partials (the residual is
  // final: this thread has passed griddepcontrol.wait, and every output
  // element is read and then written by the one thread that owns it).
  uint16_t res_pre[4] = {0, 0, 0, 0};
  if (EPI == EPI_RESIDUAL_ADD && tid < TC_EPI_THREADS && !*abort_flag) {
    const int n = nb * 128 + (tid & 127), m0 = m_begin + (tid >> 7);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int m = m0 + 2 * u, mg = mt * T + m;
      if (m < m_end && n < p.N && mg < p.M) res_pre[u] = p.residual[(size_t)mg * p.N + n];
    }
  }
  // Peers' stores land here even when this CTA gave up, so the wait does not
  // depend on the abort flag (it is bounded like every wait).
  if (!mbar_wait_cluster(&ctrl->recv_full, 0, 206)) *abort_flag = 1;

  const bool aborted = *abort_flag != 0;
  if (!aborted && tid < TC_EPI_THREADS) {
    if (EPI == EPI_RELU2_MUL) {
      const int pr = tid & 63;   // pair within the tile
      const int part = tid >> 6; // four threads share a pair, splitting tokens
      const int g0 = (pr >> 5) * 64 + (pr & 31);  // gate row in tile; up row = g0 + 32
      const int ng = nb * 128 + g0, nu = ng + 32;
      const bool row_ok = nu < N;
      uint16_t* yb = p.y + nb * 64 + (g0 >> 6) * 32 + (g0 & 31);
      const int* rg = recv + g0 - m_begin * 128;
      const int* ru = recv + (g0 + 32) - m_begin * 128;
      // Independent iterations: unrolled so their latency chains overlap.
#pragma unroll 4
      for (int m = m_begin + part; m < m_end; m += 4) {
        const int mg = mt * T + m;
        int ag = -ctrl->rsum[m], au = ag;
        for (int j = 0; j < split; ++j) {
          ag += rg[j * slot_ints + m * 128];
          au += ru[j * slot_ints + m * 128];
        }
        const float g = round_bf16(__fmul_rn(i2f_exact(ag, small_acc), ctrl->fac0[m]));
        const float u = round_bf16(__fmul_rn(i2f_exact(au, small_acc), ctrl->fac1[m]));
        const uint16_t h = relu2_mul_bf16(g, u);
        if (row_ok && mg < p.M) {
          yb[(size_t)mg * (N >> 1)] = h;
          if (p.acc_out) {
            p.acc_out[(size_t)mg * N + ng] = ag;
            p.acc_out[(size_t)mg * N + nu] = au;
          }
        }
      }
    } else {
      const int row = tid & 127;
      const int part = tid >> 7;  // two threads share a row, splitting tokens
      const int n = nb * 128 + row;
      const float wsc = seg_scale_of(p.seg, n);
      const bool row_ok = n < N;
      const int* rr = recv + row - m_begin * 128;
      // tokens in batches of 4 per thread; the batch's residuals are read before
      // any of its stores (y may be the residual buffer, which keeps the
      // compiler from moving a load above an earlier store)
      for (int m0 = m_begin + part; m0 < m_end; m0 += 8) {
        uint16_t res[4];
        if (EPI == EPI_RESIDUAL_ADD) {
          const bool first = m0 == m_begin + part;  // prefetched before the partials arrived
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int m = m0 + 2 * u, mg = mt * T + m;
            res[u] = first ? res_pre[u]
                           : ((m < m_end && row_ok && mg < p.M) ? p.residual[(size_t)mg * N + n] : (uint16_t)0);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int m = m0 + 2 * u;
          if (m >= m_end) break;
          const int mg = mt * T + m;
          int a = -ctrl->rsum[m];
          for (int j = 0; j < split; ++j) a += rr[j * slot_ints + m * 128];
          const float v = seg_uniform ? round_bf16(__fmul_rn(i2f_exact(a, small_acc), ctrl->fac0[m]))
                                      : scaled_bf16(a, wsc, ctrl->scale[m]);
          if (row_ok && mg < p.M) {
            const size_t o = (size_t)mg * N + n;
            if (p.acc_out) p.acc_out[o] = a;
            if (EPI == EPI_RESIDUAL_ADD)
              p.y[o] = residual_add_bf16(res[u], v);
            else
              p.y[o] = f32_to_bf16_bits(v);
          }
        }
      }
    }
  }

  }  // split > 1

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, ncols);
  }
}

}  // namespace bitnet
