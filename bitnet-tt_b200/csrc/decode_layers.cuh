// Persistent decode megakernel: every transformer layer of one decode step in
// a single launch.
//
// Why: at batch 32 a decode step streams ~0.5 GB of 2-bit weights but is a
// chain of ~270 small dependent operations; as separate launches each one
// pays launch, set-up (barrier init, TMEM allocation) and cold-instruction
// costs of several microseconds.  Here one CTA per SM runs the whole chain,
// the phases separated by grid barriers, with the tensor memory allocated
// once, the code hot in the instruction cache, and each BitLinear's weights
// streamed into shared memory (and unpacked into TMEM) while the previous
// phases still run.
//
// Phases of a layer (each ends with a grid barrier):
//   0 AQ_IN    act-quant(hidden, input_layernorm)           -> q_h
//   1 QKV      BitLinear(q_h) -> qkv
//   2 ATTN     RoPE + KV append + GQA attention             -> attn
//   3 AQ_ATTN  act-quant(attn, attn_sub_norm)                -> q_h
//   4 O        BitLinear(q_h) + hidden                      -> hidden
//   5 AQ_POST  act-quant(hidden, post_attention_layernorm)  -> q_h
//   6 GU       BitLinear(q_h), ReLU^2(gate) * up             -> mid
//   7 AQ_FFN   act-quant(mid, ffn_sub_norm)                  -> q_f
//   8 DOWN     BitLinear(q_f) + hidden                      -> hidden
// The arithmetic of every phase is the code of the standalone kernels
// (aq_row_vec, attn_unit, the tcgen05 contraction and its epilogue), so the
// results are bit-identical to the per-operation path.
//
// Warp roles (512 threads, one CTA per SM):
//   warps 0-7   workers: act-quant rows, attention units, BitLinear
//               epilogues, grid barriers (named barrier 1 over 256 threads);
//   warps 8-11  unpackers: packed 2-bit weights (shared memory) -> int8 codes
//               in a ring of TMEM A buffers (warp w owns TMEM lane quarter w % 4);
//   warps 12-14 MMA issuers (lane 0): tcgen05.mma kind::i8 into accumulators
//               D_0..D_2, one per issuer;
//   warp 15     producer (one lane per ring slot): bulk copies of weights
//               (ahead, across phase boundaries, as far as the ring allows) and
//               of the activation codes (once the grid barrier that produced
//               them has passed).
// BitLinear work units are (row tile of 128, K split); a split-K unit adds its
// int32 partial sums to a global scratch tile with red.add, and the last unit
// of the tile to finish (an arrival counter) applies the epilogue and clears
// the scratch.
//
// Every wait is bounded.  A wait that runs out records the device error, sets
// a global abort flag that every other wait of every CTA polls, and all roles
// leave their loops; copies in flight and MMAs land before the CTA exits and
// frees its tensor memory.
#pragma once
#include "act_quant.cuh"
#include "attention.cuh"
#include "common.cuh"
#include "epilogue.cuh"

namespace bitnet {

constexpr int MK_WORKER_WARPS = 8;
constexpr int MK_WORKERS = MK_WORKER_WARPS * 32;
constexpr int MK_UNPACK_WARP0 = 8;
constexpr int MK_MMA_WARP0 = 12;
constexpr int MK_PRODUCER_WARP = 15;
// 16 warps: 4 per SM sub-partition, so each thread may use 128 registers (a
// 17th warp would put 5 warps on one sub-partition and cap them at 96)
constexpr int MK_THREADS = 16 * 32;
constexpr int MK_NSLOT = 12;
constexpr int MK_STAGE_CHUNKS = 4;                         // 4 x 64 = 256 K per stage
constexpr int MK_NACC = 3;                                 // MMA issuers / accumulators
constexpr int MK_NB = 6;                                   // TMEM A buffers of 64 columns
constexpr int MK_MAX_T = 32;
constexpr int MK_WSLOT = MK_STAGE_CHUNKS * 2048;           // packed weights of a stage
constexpr int MK_XSLOT = MK_STAGE_CHUNKS * 64 * MK_MAX_T;  // activation codes of a stage
constexpr int MK_SLOT = MK_WSLOT + MK_XSLOT;
constexpr int MK_CTRL_BYTES = 2048;
constexpr int MK_BAR = 1;                                  // named barrier of the workers
constexpr int MK_PHASES = 9;
constexpr long long MK_POLL_GRACE = 20000;                 // cycles before a wait polls the abort flag

enum MkPhase { PH_AQ_IN = 0, PH_QKV, PH_ATTN, PH_AQ_ATTN, PH_O, PH_AQ_POST, PH_GU, PH_AQ_FFN, PH_DOWN };
__host__ __device__ constexpr int mk_bl_phase(int bp) {
  return bp == 0 ? PH_QKV : (bp == 1 ? PH_O : (bp == 2 ? PH_GU : PH_DOWN));
}

struct MkLayer {
  const uint8_t* w[4];           // packed weights: qkv, o, gate_up (interleaved), down
  bitnet_segments_dev seg[4];
  const uint16_t* gamma[4];      // input_layernorm, attn_sub_norm, post_attention_layernorm, ffn_sub_norm
  uint16_t* k_cache;
  uint16_t* v_cache;
};

struct MkBl {       // one BitLinear of the layer (same shape in every layer)
  int N, K, KC;     // output rows, input features, K chunks of 64
  int NT, S;        // row tiles of 128, K splits
  int epi;          // EPI_*
};

struct MkParams {
  const MkLayer* layers;  // device array [L]
  int L, B, T;
  float eps;
  MkBl bl[4];             // qkv, o, gate_up, down
  uint16_t* hidden;       // [B][H] bf16, in / out
  uint16_t* qkv;          // [B][QKV]
  uint16_t* attn;         // [B][n_heads * 128]
  uint16_t* mid;          // [B][F] (ReLU^2(gate) * up)
  int8_t* q_h;            // codes of the current K = H (or n_heads*128) activation, tile T x Kp
  float* s_h;
  int32_t* rs_h;
  int8_t* q_f;            // codes of the FFN activation
  float* s_f;
  int32_t* rs_f;
  int32_t* acc_ws;        // [max NT][T][128] split-K partial sums, zero between uses
  int* tile_cnt;          // [max NT] split-K arrival counters, zero between uses
  unsigned* sync_ctr;     // grid barrier arrivals (zeroed before each launch)
  int* abort_flag;        // set when any wait of any CTA runs out (zeroed before each launch)
  AttnParams att;         // k_cache / v_cache are taken from the layer
  int att_units;          // B * n_kv * att.nsplit
};

struct MkCtrl {
  uint64_t w_full[MK_NSLOT];
  uint64_t x_full[MK_NSLOT];
  uint64_t slot_free[MK_NSLOT];
  uint64_t a_full[MK_NB];
  uint64_t a_empty[MK_NB];
  uint64_t d_final;
  uint64_t d_empty;
  uint64_t mma_done[MK_NACC];
  uint32_t tmem_base;
  int att_flag[2];
  int last_flag;
  int stop;               // workers: CTA-uniform abort decision
  unsigned sync_seen;     // grid barriers passed (written by worker 0, read by the producer)
  double red_d[8];
  float red_f[8];
  int red_i[8];
  float scale[MK_MAX_T];
  int rsum[MK_MAX_T];
  float fac0[MK_MAX_T];
  float fac1[MK_MAX_T];
};
static_assert(sizeof(MkCtrl) <= MK_CTRL_BYTES, "control block");

// Attention (two units at a time, one per group of 4 workers) uses the weight
// ring for its K / V tiles: the producer does not refill the ring between the
// end of the QKV MMAs and the end of the attention phase.
// Shared memory: control | ring | epilogue exchange | attention small regions x 2.
static_assert(2 * ATT_TILES_BYTES <= MK_NSLOT * MK_SLOT, "attention tiles fit the ring");
constexpr int MK_XCHG_BYTES = 2 * 2 * 32 * 16 * 4;  // gate/up exchange of the ReLU^2 epilogue
__host__ __device__ __forceinline__ size_t mk_smem_bytes(int G) {
  return (size_t)MK_CTRL_BYTES + (size_t)MK_NSLOT * MK_SLOT + MK_XCHG_BYTES + 2 * att_small_bytes(G);
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_acq_rel_add_s32(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release_cta_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_cta_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_s32(int32_t* p, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool mk_aborted(const MkParams& p) {
  return *reinterpret_cast<volatile const int*>(p.abort_flag) != 0;
}
__device__ __forceinline__ void mk_raise(const MkParams& p, int site) {
  record_error(DEV_ERR_TIMEOUT, site);
  atomicExch(p.abort_flag, 1);
}
// Bounded mbarrier wait that also gives up when another CTA aborted.  After a
// few polls it backs off, so that waiting roles leave the issue slots to the
// warps doing work.
__device__ __forceinline__ bool mk_wait(const MkParams& p, uint64_t* bar, uint32_t parity, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  int polls = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++polls > 4) __nanosleep(64);
    const long long dt = clock64() - t0;
    if (dt > MK_POLL_GRACE && mk_aborted(p)) return false;
    if (dt > kSpinLimitCycles) {
      mk_raise(p, site);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// The CTA's BitLinear stages, in the order every role walks them: layers,
// then the four BitLinears, then this CTA's units (u = blockIdx.x + i * grid),
// then the unit's stages of up to 4 K chunks.
struct StageIter {
  int l, bp, u, s;
  int nt, kc0, kc_end, nstages;
  bool valid;
};
__device__ __forceinline__ void si_settle(StageIter& it, const MkParams& p) {
  while (it.l < p.L) {
    const MkBl& bl = p.bl[it.bp];
    if (it.u < bl.NT * bl.S) {
      it.nt = it.u % bl.NT;
      const int ks = it.u / bl.NT;
      it.kc0 = (ks * bl.KC) / bl.S;
      it.kc_end = ((ks + 1) * bl.KC) / bl.S;
      it.nstages = (it.kc_end - it.kc0 + MK_STAGE_CHUNKS - 1) / MK_STAGE_CHUNKS;
      it.valid = true;
      return;
    }
    it.u = blockIdx.x;
    it.s = 0;
    if (++it.bp == 4) {
      it.bp = 0;
      ++it.l;
    }
  }
  it.valid = false;
}
__device__ __forceinline__ void si_init(StageIter& it, const MkParams& p) {
  it.l = 0;
  it.bp = 0;
  it.u = blockIdx.x;
  it.s = 0;
  si_settle(it, p);
}
__device__ __forceinline__ void si_next(StageIter& it, const MkParams& p) {
  if (++it.s < it.nstages) return;
  it.s = 0;
  it.u += gridDim.x;
  si_settle(it, p);
}
__device__ __forceinline__ int si_chunk0(const StageIter& it) { return it.kc0 + it.s * MK_STAGE_CHUNKS; }
__device__ __forceinline__ int si_nch(const StageIter& it) {
  return min(MK_STAGE_CHUNKS, it.kc_end - si_chunk0(it));
}

// ---------------------------------------------------------------------------
// producer: lane j (< MK_NSLOT) owns ring slot j, i.e. the stages g with
// g % MK_NSLOT == j (a thread's bulk copies complete one after another, so
// the slots are filled in parallel).  Weights go ahead as far as the slot
// allows, except that no weights are written into the ring between the QKV
// MMAs and the end of the attention phase (attention keeps its tiles there); the
// activation codes of a phase go once its input's grid barrier has passed.
__device__ __forceinline__ void si_next_mine(StageIter& it, const MkParams& p, int& g) {
  for (int i = 0; i < MK_NSLOT && it.valid; ++i) {
    si_next(it, p);
    ++g;
  }
}
__device__ void mk_producer(const MkParams& p, MkCtrl* c, uint8_t* ring, int lane) {
  StageIter wi, ai;
  si_init(wi, p);
  si_init(ai, p);
  int gw = 0, ga = 0;  // global stage index of the next weight / activation copy of this lane
  for (int i = 0; i < lane && wi.valid; ++i) {
    si_next(wi, p);
    si_next(ai, p);
    ++gw;
    ++ga;
  }
  unsigned seen = 0;  // grid barriers known to have passed
  const uint64_t policy = l2_policy_evict_first();
  uint8_t* slot_w = ring + (size_t)lane * MK_SLOT;
  long long idle = clock64();
  bool stop = false;
  while (ai.valid && !stop) {
    bool prog = false;
    if (wi.valid && gw - ga < MK_NSLOT) {
      // The ring holds attention tiles from grid barrier l*9 + 2 to l*9 + 3:
      // weights consumed after the attention of layer l (o, gate_up, down of
      // layer l; qkv of layer l + 1) go in only once it has ended.
      const unsigned wneed = wi.bp != 0   ? (unsigned)(wi.l * MK_PHASES + PH_AQ_ATTN)
                             : wi.l > 0 ? (unsigned)((wi.l - 1) * MK_PHASES + PH_AQ_ATTN)
                                        : 0u;
      if (seen < wneed) seen = ld_acquire_cta_u32(&c->sync_seen);
      if (seen >= wneed && (gw < MK_NSLOT || mbar_test_wait(&c->slot_free[lane], ((gw / MK_NSLOT) + 1) & 1))) {
        if (wneed) fence_proxy_async_smem();  // attention's reads of the ring precede the copy
        const int nch = si_nch(wi);
        const uint8_t* src = p.layers[wi.l].w[wi.bp] + ((size_t)wi.nt * p.bl[wi.bp].KC + si_chunk0(wi)) * 2048u;
        mbar_arrive_expect_tx(&c->w_full[lane], (uint32_t)(nch * 2048));
        bulk_g2s_stream(slot_w, src, (uint32_t)(nch * 2048), &c->w_full[lane], policy);
        si_next_mine(wi, p, gw);
        prog = true;
      }
    }
    if (ga < gw) {
      // the activation codes of phase (l, ph) exist once grid barrier l * 9 + ph has passed
      const unsigned need = (unsigned)(ai.l * MK_PHASES + mk_bl_phase(ai.bp));
      if (seen < need) seen = ld_acquire_cta_u32(&c->sync_seen);
      if (seen >= need) {
        fence_proxy_async_global();
        const int nch = si_nch(ai);
        const int8_t* q = ai.bp == 3 ? p.q_f : p.q_h;
        mbar_arrive_expect_tx(&c->x_full[lane], (uint32_t)(nch * 64 * p.T));
        bulk_g2s(slot_w + MK_WSLOT, q + (size_t)si_chunk0(ai) * 64 * p.T, (uint32_t)(nch * 64 * p.T),
                 &c->x_full[lane]);
        si_next_mine(ai, p, ga);
        prog = true;
      }
    }
    if (prog) {
      idle = clock64();
    } else {
      __nanosleep(32);
      const long long dt = clock64() - idle;
      if (dt > MK_POLL_GRACE && mk_aborted(p)) stop = true;
      if (dt > kSpinLimitCycles) {
        mk_raise(p, 600);
        stop = true;
      }
    }
  }
  if (stop) {  // this lane's copies in flight land before shared memory is released
    for (int g = ga - MK_NSLOT; g < gw; g += MK_NSLOT)
      if (g >= 0) mbar_wait(&c->w_full[lane], (g / MK_NSLOT) & 1, 601);
    for (int g = ga - MK_NSLOT; g < ga; g += MK_NSLOT)
      if (g >= 0) mbar_wait(&c->x_full[lane], (g / MK_NSLOT) & 1, 602);
  }
}

// ---------------------------------------------------------------------------
// unpacker warp (TMEM lane quarter `quarter`)
__device__ void mk_unpack(const MkParams& p, MkCtrl* c, const uint8_t* ring, uint32_t tbase, int quarter, int lane) {
  StageIter it;
  si_init(it, p);
  const int row = quarter * 32 + lane;
  for (int g = 0; it.valid; ++g, si_next(it, p)) {
    const int slot = g % MK_NSLOT, b = g % MK_NB;
    bool ok = true;
    if (g >= MK_NB) ok = mk_wait(p, &c->a_empty[b], ((g / MK_NB) + 1) & 1, 610);
    if (ok) ok = mk_wait(p, &c->w_full[slot], (g / MK_NSLOT) & 1, 611);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      const uint8_t* wsm = ring + (size_t)slot * MK_SLOT;
      const uint32_t tst = tbase + ((uint32_t)(quarter * 32) << 16) + b * 64;
      const int nch = si_nch(it);
      for (int ch = 0; ch < nch; ++ch) {
        const uint4 v = *reinterpret_cast<const uint4*>(wsm + ch * 2048 + row * 16);
        uint32_t o[16];
        unpack16(v.x, o[0], o[1], o[2], o[3]);
        unpack16(v.y, o[4], o[5], o[6], o[7]);
        unpack16(v.z, o[8], o[9], o[10], o[11]);
        unpack16(v.w, o[12], o[13], o[14], o[15]);
        tmem_st16(tst + ch * 16, o);
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&c->a_full[b]);
    if (!ok) break;
  }
}

// ---------------------------------------------------------------------------
// MMA issuer `iss` (one thread): K steps kk = iss, iss + 4, ... of every stage
// into its own accumulator D_iss.
__device__ void mk_mma(const MkParams& p, MkCtrl* c, uint8_t* ring, uint32_t tbase, int iss) {
  StageIter it;
  si_init(it, p);
  const uint32_t idesc = idesc_i8_s32(128, p.T);
  const uint32_t d = tbase + MK_NB * 64 + iss * p.T;
  int ui = 0;
  bool first = true;
  for (int g = 0; it.valid; ++g) {
    const int slot = g % MK_NSLOT, b = g % MK_NB;
    if (it.s == 0) {
      if (ui > 0 && !mk_wait(p, &c->d_empty, (ui - 1) & 1, 620)) break;
      first = true;
    }
    if (!mk_wait(p, &c->a_full[b], (g / MK_NB) & 1, 621)) break;
    if (!mk_wait(p, &c->x_full[slot], (g / MK_NSLOT) & 1, 622)) break;
    tc_fence_after();
    const uint32_t a_base = tbase + b * 64;
    const uint32_t b_base = smem_u32(ring + (size_t)slot * MK_SLOT + MK_WSLOT);
    const int ksteps = 2 * si_nch(it);
    for (int kk = iss; kk < ksteps; kk += MK_NACC) {
      const uint64_t bdesc = smem_desc_kmajor(b_base + kk * 32 * p.T, 16 * p.T, 128);
      mma_i8_ts(d, a_base + kk * 8, bdesc, idesc, first ? 0u : 1u);
      first = false;
    }
    tc_commit(&c->a_empty[b]);
    tc_commit(&c->slot_free[slot]);
    const bool last = it.s == it.nstages - 1;
    si_next(it, p);
    if (last) {
      tc_commit(&c->d_final);
      ++ui;
    }
  }
  // every MMA this thread issued has completed before tensor memory is freed
  tc_commit(&c->mma_done[iss]);
  mbar_wait(&c->mma_done[iss], 0, 623);
}

// ---------------------------------------------------------------------------
// workers
__device__ __forceinline__ void mk_bar() { named_bar_sync(MK_BAR, MK_WORKERS); }

// CTA-uniform "keep going" after a step whose threads may disagree.
__device__ __forceinline__ bool mk_uniform_ok(MkCtrl* c, bool ok, int t) {
  if (!ok) c->stop = 1;
  mk_bar();
  const bool r = c->stop == 0;
  mk_bar();
  return r;
}

__device__ __forceinline__ void mk_aq(const MkParams& p, const uint16_t* x, int K, const uint16_t* gamma, int8_t* q, float* s,
                      int32_t* rs, MkCtrl* c, int t) {
  const AqScratch sc{c->red_d, c->red_f, c->red_i};
  const int Kp = (K + 63) / 64 * 64;
  for (int m = blockIdx.x; m < p.T; m += gridDim.x) {
    uint4 gr[AQ_MAXC];
    aq_load_gamma(gr, gamma, K, t);
    aq_row_vec<MK_BAR>(x, p.B, K, K, gamma != nullptr, gr, p.eps, q, s, rs, nullptr, p.T, Kp, m, sc, t);
  }
}

// This group's attention units (group gi of two; units gi, gi + 2, ... of the
// CTA's share).
template <int G>
__device__ __forceinline__ bool mk_attn(const MkParams& p, const MkLayer& lw, const AttnSmem& sm,
                                        uint32_t& tiles_done, int gi, int tg) {
  AttnParams a = p.att;
  a.k_cache = lw.k_cache;
  a.v_cache = lw.v_cache;
  for (int u = blockIdx.x * 2 + gi; u < p.att_units; u += gridDim.x * 2) {
    const int b = u % p.B;
    const int r = u / p.B;
    if (!attn_unit<G>(a, b, r % a.n_kv, r / a.n_kv, sm, tiles_done, tg, 2 + gi)) return false;
  }
  return true;
}

// Epilogue of one finished tile (values of this thread: row r, tokens
// c0 .. c0 + 15 in v[]).  Same arithmetic as bitlinear_tc_kernel.
__device__ __forceinline__ void mk_finish(const MkParams& p, const MkBl& bl, const bitnet_segments_dev& seg, int bp, int nt, int c0,
                          bool has_cols, const int (&v)[16], int r, MkCtrl* c, int* xchg, int t) {
  const int n = nt * 128 + r;
  const int N = bl.N;
  if (bl.epi == EPI_RELU2_MUL) {
    // rows of a 64-row group: [32 gate | 32 up]; lane quarters 0 / 2 hold gate
    // rows, 1 / 3 the matching up rows
    const int w = t >> 5, lane = t & 31, quarter = w & 3, half = w >> 2;
    int* slot = xchg + (((quarter >> 1) * 2 + half) * 32 + lane) * 16;
    if ((quarter & 1) && has_cols) {
#pragma unroll
      for (int j = 0; j < 16; ++j) slot[j] = v[j];
    }
    mk_bar();
    if (!(quarter & 1) && has_cols) {
      const int gcol = nt * 64 + (quarter >> 1) * 32 + lane;  // output column
      const bool row_ok = n + 32 < N;
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int m = c0 + j;
        const int ag = v[j] - c->rsum[m], au = slot[j] - c->rsum[m];
        const float gv = round_bf16(__fmul_rn((float)ag, c->fac0[m]));
        const float uv = round_bf16(__fmul_rn((float)au, c->fac1[m]));
        if (row_ok && m < p.B) p.mid[(size_t)m * (N >> 1) + gcol] = relu2_mul_bf16(gv, uv);
      }
    }
    mk_bar();  // the exchange area is reused by the next tile
    return;
  }
  if (!has_cols || n >= N) return;
  const float wsc = seg_scale_of(seg, n);
  const bool uniform = seg_scale_of(seg, nt * 128) == seg_scale_of(seg, min(N, nt * 128 + 128) - 1);
  uint16_t* y = bp == 0 ? p.qkv : p.hidden;
  const int mend = min(16, p.B - c0);
  // residual rows first, all in flight at once (one memory round trip)
  uint16_t res[16];
  if (bl.epi == EPI_RESIDUAL_ADD) {
#pragma unroll
    for (int j = 0; j < 16; ++j) res[j] = j < mend ? y[(size_t)(c0 + j) * N + n] : (uint16_t)0;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j < mend) {
      const int m = c0 + j;
      const int a = v[j] - c->rsum[m];
      const float val = uniform ? round_bf16(__fmul_rn((float)a, c->fac0[m])) : scaled_bf16(a, wsc, c->scale[m]);
      y[(size_t)m * N + n] = bl.epi == EPI_RESIDUAL_ADD ? residual_add_bf16(res[j], val) : f32_to_bf16_bits(val);
    }
  }
}

// Epilogues of this CTA's units of BitLinear bp.  Returns false on abort.
__device__ __forceinline__ bool mk_bl_epilogue(const MkParams& p, int bp, const MkLayer& lw, MkCtrl* c, uint32_t tmem_d, int& ui,
                               int* xchg, int t) {
  const MkBl& bl = p.bl[bp];
  const float* srow = bp == 3 ? p.s_f : p.s_h;
  const int32_t* rsrow = bp == 3 ? p.rs_f : p.rs_h;
  const int w = t >> 5, lane = t & 31, quarter = w & 3, half = w >> 2;
  const int r = quarter * 32 + lane;
  const int c0 = half * 16;
  const bool has_cols = c0 < p.T;
  for (int u = blockIdx.x; u < bl.NT * bl.S; u += gridDim.x) {
    const int nt = u % bl.NT, ks = u / bl.NT;
    const int kcb = (ks * bl.KC) / bl.S, kce = ((ks + 1) * bl.KC) / bl.S;
    const int used_acc = min(MK_NACC, 2 * (kce - kcb));
    // per-token factors (overlap the MMAs)
    if (t < p.T) {
      const float s = srow[t];
      const float sc0 = bl.epi == EPI_RELU2_MUL ? lw.seg[bp].scale[0] : seg_scale_of(lw.seg[bp], nt * 128);
      c->scale[t] = s;
      c->rsum[t] = rsrow[t];
      c->fac0[t] = __fdiv_rn(sc0, s);
      if (bl.epi == EPI_RELU2_MUL) c->fac1[t] = __fdiv_rn(lw.seg[bp].scale[1], s);
    }
    bool ok = mk_wait(p, &c->d_final, ui & 1, 630);
    ok = mk_uniform_ok(c, ok, t);  // also publishes the factors
    if (!ok) return false;
    tc_fence_after();
    int v[16];
    if (has_cols) {
      const uint32_t base = tmem_d + ((uint32_t)(quarter * 32) << 16) + c0;
      uint32_t a[16];
      tmem_ld16(base, a);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (int)a[j];
      for (int i = 1; i < used_acc; ++i) {
        tmem_ld16(base + i * p.T, a);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += (int)a[j];
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&c->d_empty);  // the next unit's MMAs may overwrite D
    ++ui;
    bool finish = bl.S == 1;
    if (!finish) {
      int32_t* ws = p.acc_ws + (size_t)nt * p.T * 128;
      if (has_cols) {
#pragma unroll
        for (int j = 0; j < 16; ++j) red_add_s32(ws + (c0 + j) * 128 + r, v[j]);
      }
      mk_bar();  // the CTA's additions precede worker 0's release below
      if (t == 0) {
        const int old = atom_acq_rel_add_s32(p.tile_cnt + nt, 1);
        const int last = old == bl.S - 1;
        if (last) atomicExch(p.tile_cnt + nt, 0);  // ready for the next BitLinear
        c->last_flag = last;
      }
      mk_bar();  // worker 0's acquire precedes every worker's reads below
      finish = c->last_flag != 0;
      if (finish) {
        if (has_cols) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = __ldcg(ws + (c0 + j) * 128 + r);
            __stcg(ws + (c0 + j) * 128 + r, 0);
          }
        }
      }
    }
    if (finish) mk_finish(p, bl, lw.seg[bp], bp, nt, c0, has_cols, v, r, c, xchg, t);
    mk_bar();  // factors and flags are rewritten by the next unit
  }
  return true;
}

// Grid barrier number k (1-based) among the workers of every CTA.  Returns
// false (CTA-uniform) when the run is aborting.
__device__ bool mk_grid_sync(const MkParams& p, MkCtrl* c, int k, int t) {
  fence_proxy_async_global();  // this thread's stores are read by other CTAs' bulk copies
  mk_bar();
  if (t == 0) {
    red_release_add_u32(p.sync_ctr, 1u);  // cumulative over the CTA's writes (bar.sync above)
    const unsigned target = (unsigned)k * gridDim.x;
    const long long t0 = clock64();
    while (ld_acquire_gpu(p.sync_ctr) < target) {
      __nanosleep(32);
      const long long dt = clock64() - t0;
      if (dt > MK_POLL_GRACE && mk_aborted(p)) {
        c->stop = 1;
        break;
      }
      if (dt > kSpinLimitCycles) {
        mk_raise(p, 640);
        c->stop = 1;
        break;
      }
    }
    st_release_cta_u32(&c->sync_seen, (unsigned)k);  // lets the producer fetch this phase's inputs
  }
  mk_bar();
  return c->stop == 0;
}

template <int G>
__device__ void mk_worker(const MkParams& p, MkCtrl* c, uint8_t* ring, int* xchg, uint8_t* att_region,
                          uint32_t tmem_d, int t) {
  const int gi = t >> 7, tg = t & 127;  // attention group of this thread
  const AttnSmem asm_ = att_carve(ring + (size_t)gi * ATT_TILES_BYTES, att_region + gi * att_small_bytes(G), G,
                                  &c->att_flag[gi]);
  uint32_t tiles_done = 0;
  int ui = 0, nsync = 0;
  const int attn_k = p.att.n_heads * ATT_D;
  for (int l = 0; l < p.L; ++l) {
    const MkLayer& lw = p.layers[l];
    for (int ph = 0; ph < MK_PHASES; ++ph) {
      bool ok = true;
      if (ph == PH_ATTN) {
        fence_proxy_async_smem();  // earlier generic reads of the ring precede the tiles' bulk copies
        ok = mk_attn<G>(p, lw, asm_, tiles_done, gi, tg);
        ok = mk_uniform_ok(c, ok, t);
      } else if (ph == PH_QKV || ph == PH_O || ph == PH_GU || ph == PH_DOWN) {
        const int bp = ph == PH_QKV ? 0 : (ph == PH_O ? 1 : (ph == PH_GU ? 2 : 3));
        ok = mk_bl_epilogue(p, bp, lw, c, tmem_d, ui, xchg, t);
      } else {
        const uint16_t* x = ph == PH_AQ_ATTN ? p.attn : (ph == PH_AQ_FFN ? p.mid : p.hidden);
        const int K = ph == PH_AQ_ATTN ? attn_k : (ph == PH_AQ_FFN ? p.bl[3].K : p.bl[0].K);
        const int gsel = ph == PH_AQ_IN ? 0 : (ph == PH_AQ_ATTN ? 1 : (ph == PH_AQ_POST ? 2 : 3));
        const bool ffn = ph == PH_AQ_FFN;
        mk_aq(p, x, K, lw.gamma[gsel], ffn ? p.q_f : p.q_h, ffn ? p.s_f : p.s_h, ffn ? p.rs_f : p.rs_h, c, t);
      }
      if (!ok) {
        if (t == 0) atomicExch(p.abort_flag, 1);
        return;
      }
      if (l == p.L - 1 && ph == MK_PHASES - 1) return;  // the launch boundary ends the last phase
      if (!mk_grid_sync(p, c, ++nsync, t)) return;
    }
  }
}

template <int G>
__global__ void __launch_bounds__(MK_THREADS) decode_layers_kernel(const MkParams p) {
  extern __shared__ __align__(1024) uint8_t smem_mk[];
  MkCtrl* c = reinterpret_cast<MkCtrl*>(smem_mk);
  uint8_t* ring = smem_mk + MK_CTRL_BYTES;
  int* xchg = reinterpret_cast<int*>(ring + (size_t)MK_NSLOT * MK_SLOT);
  uint8_t* att_region = ring + (size_t)MK_NSLOT * MK_SLOT + MK_XCHG_BYTES;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < MK_NSLOT; ++i) {
      mbar_init(&c->w_full[i], 1);
      mbar_init(&c->x_full[i], 1);
      mbar_init(&c->slot_free[i], MK_NACC);
    }
    for (int b = 0; b < MK_NB; ++b) {
      mbar_init(&c->a_full[b], 4);
      mbar_init(&c->a_empty[b], MK_NACC);
    }
    mbar_init(&c->d_final, MK_NACC);
    mbar_init(&c->d_empty, MK_WORKER_WARPS);
    for (int i = 0; i < MK_NACC; ++i) mbar_init(&c->mma_done[i], 1);
    for (int gi = 0; gi < 2; ++gi) {
      const AttnSmem a = att_carve(ring, att_region + gi * att_small_bytes(G), G, &c->att_flag[gi]);
      for (int i = 0; i < ATT_WARPS * ATT_NBUF; ++i) mbar_init(&a.bars[i], ATT_BAR_COUNT);
      c->att_flag[gi] = 0;
    }
    c->last_flag = 0;
    c->stop = 0;
    c->sync_seen = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&c->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = c->tmem_base;

  if (warp == MK_PRODUCER_WARP) {
    if (lane < MK_NSLOT) mk_producer(p, c, ring, lane);
  } else if (warp >= MK_MMA_WARP0) {
    if (lane == 0) mk_mma(p, c, ring, tbase, warp - MK_MMA_WARP0);
  } else if (warp >= MK_UNPACK_WARP0) {
    mk_unpack(p, c, ring, tbase, warp - MK_UNPACK_WARP0, lane);
  } else {
    mk_worker<G>(p, c, ring, xchg, att_region, tbase + MK_NB * 64, tid);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace bitnet
