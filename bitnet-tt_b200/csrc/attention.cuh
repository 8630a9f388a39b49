// GQA decode attention with fused rotary embedding and KV-cache append.
//
// Work unit (b, g, s): the G = n_heads / n_kv_heads query heads that share KV
// head g (HF repeat_kv grouping: query head h uses KV head h / G) of sequence b,
// over part s of its L = positions[b] + 1 keys.  The grid has `nsplit` units
// per (b, g), chosen on the host from B * n_kv_heads and max_ctx
// (att_grid_splits); every sequence is cut into parts of the same length,
// ceil(max_ctx / nsplit) keys in whole 16-key tiles (att_parts), so a short
// context takes fewer units than a long one, and units past a sequence's last
// part return at once.  So a long context over many sequences runs as one
// long unit per (b, g), and a few sequences spread over the GPU.  A unit runs
// on 4 warps:
//   1. RoPE (HF half-split convention, bf16 op-by-op like transformers'
//      apply_rotary_pos_emb on bf16 tensors):
//        out[i]    = bf16(bf16(x[i] * cos_i)    + bf16(-x[i+64] * sin_i))
//        out[i+64] = bf16(bf16(x[i+64] * cos_i) + bf16( x[i]    * sin_i))
//      on the G query heads and the new key; the unit whose range holds the
//      new position writes the rotated key and the value to row positions[b].
//   2. Warp w takes the 16-key tiles w, w + 4, ... of the range: the tile's K
//      and V rows (4 KB each, contiguous in the cache) arrive by per-lane
//      16-byte cp.async into an XOR-swizzled double buffer of the warp's own,
//      the first two issued before the RoPE so that their latency overlaps it.
//      Per tile, S^T = Q K^T and O^T += V^T P^T run on mma.sync m16n8k16 (K and
//      V through ldmatrix; P from the score fragments as a bf16 hi + lo pair),
//      with an online softmax in base 2 across the tiles (see attn_unit).  The
//      tile holding the new position takes the rotated key and the value from
//      shared memory, not from the cache row being written.
//   3. The warps' states merge in shared memory.  With one active unit per
//      (b, g) the result is normalised and written; otherwise each unit writes
//      (max, sum, unnormalised accumulator) to the workspace and the last unit
//      of (b, g) to finish (a counter in the workspace, reset by that unit)
//      merges the parts.
#pragma once
#include <algorithm>

#include "common.cuh"

namespace bitnet {

constexpr int ATT_THREADS = 128;                     // one unit = 4 warps
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int ATT_D = 128;
constexpr int ATT_MAX_G = 8;
constexpr int ATT_TILE = 16;                         // keys per tile
constexpr int ATT_NBUF = 2;                          // tiles in flight per warp
constexpr int ATT_TILE_BYTES = ATT_TILE * ATT_D * 2; // K (or V) of one tile
constexpr int ATT_MIN_SPLIT = 256;                   // keys of max_ctx per grid unit, at least
// The split-count model (att_grid_splits).  Three 66 KB units fit on an SM,
// so a B200 (148 SMs) holds 444 at once; a unit costs its keys plus about
// 128 keys' worth of fixed work (RoPE, pipeline fill, the partial-state round
// trip and the merge).  Fewer, longer units pay that less often: at 256
// sequences x 4K keys one unit per (b, g) beats 16 units of 256 keys by a
// fifth of the decode step, and 7 units of 620 keys by a sixth.
constexpr int ATT_SLOTS = 444;
constexpr int ATT_UNIT_COST = 128;
constexpr int ATT_TILES_BYTES = ATT_WARPS * ATT_NBUF * 2 * ATT_TILE_BYTES;  // 64 KB
constexpr int ATT_QROW = 136;                        // bf16 per query row in shared memory (padded)

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
  int prefetch;     // 1: units ask L2 for their K / V rows before griddepcontrol.wait
};

// K / V bytes a launch may touch, up to which the units' early L2 requests pay:
// at config-2 contexts (32 sequences x 5 KV heads x 192 keys, 15.7 MB) they took
// the decode step from 1520 to 1508 us; at config-4 contexts (hundreds of MB per
// launch, more than L2 holds) they slowed the attention from 238 to 267 us per
// launch (256 sequences) and from 72.7 to 81.5 us (64 sequences).
constexpr size_t ATT_PREFETCH_MAX_BYTES = (size_t)32 << 20;
inline int att_prefetch_pays(int B, int n_kv, int max_ctx) {
  return (size_t)B * n_kv * max_ctx * ATT_D * 2 * 2 <= ATT_PREFETCH_MAX_BYTES ? 1 : 0;
}

__host__ __device__ __forceinline__ int att_part_floats(int G) { return 2 * G + G * ATT_D; }

// Units per (b, g) in the grid: the s in 1 .. ceil(max_ctx / 256) with the
// least modelled time, waves x unit length =
// ceil(B n_kv s / ATT_SLOTS) x (ceil(max_ctx / s) + ATT_UNIT_COST), the
// smallest s on a tie.  A wave that is barely begun costs a whole unit, so the
// model avoids unit counts just past a multiple of the slots.
inline int att_grid_splits(int B, int n_kv, int max_ctx) {
  const long long pairs = (long long)B * n_kv;
  const int smax = (int)std::max<long long>(1, ((long long)max_ctx + ATT_MIN_SPLIT - 1) / ATT_MIN_SPLIT);
  int best_s = 1;
  long long best = -1;
  for (int s = 1; s <= smax; ++s) {
    const long long waves = (pairs * s + ATT_SLOTS - 1) / ATT_SLOTS;
    const long long cost = waves * (((long long)max_ctx + s - 1) / s + ATT_UNIT_COST);
    if (best < 0 || cost < best) {
      best = cost;
      best_s = s;
    }
  }
  return best_s;
}

// The parts of a sequence of L keys (1 <= L <= max_ctx): span =
// ceil(max_ctx / nsplit) rounded up to a whole tile, nparts = ceil(L / span)
// <= nsplit; every part is non-empty and part nparts - 1 holds key L - 1.  One
// span for all sequences (not ceil(L / nparts) per sequence) gives a short
// context fewer units, each of which costs about 128 keys of fixed work:
// measured 1.8% faster decode steps at 32 and 128 ragged 4K-contexts per GPU.
__host__ __device__ __forceinline__ void att_parts(int L, int nsplit, int max_ctx, int& nparts, int& span) {
  span = ((max_ctx + nsplit - 1) / nsplit + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
  nparts = (L + span - 1) / span;
}

// Shared memory of one unit besides its tiles: rotated queries bf16
// [G][ATT_QROW] | new key, new value (bf16) | mbarriers [warp][buffer].
__host__ __device__ __forceinline__ size_t att_small_bytes(int G) {
  return ((size_t)G * ATT_QROW * 2 + 2 * ATT_D * 2 + ATT_WARPS * ATT_NBUF * 8 + 127) / 128 * 128;
}
__host__ __device__ __forceinline__ size_t att_smem_bytes(int G) { return ATT_TILES_BYTES + att_small_bytes(G); }

struct AttnSmem {
  uint8_t* tiles;  // ATT_TILES_BYTES, 128-byte aligned
  uint16_t* qb;
  uint16_t* knew;
  uint16_t* vnew;
  uint64_t* bars;  // [warp][buffer], count 32 (one cp.async arrival per lane)
  int* flag;       // one int: abort / "this unit merges"
};

__device__ __forceinline__ AttnSmem att_carve(uint8_t* tiles, uint8_t* small, int G, int* flag) {
  AttnSmem s;
  s.tiles = tiles;
  s.qb = reinterpret_cast<uint16_t*>(small);
  s.knew = s.qb + G * ATT_QROW;
  s.vnew = s.knew + ATT_D;
  s.bars = reinterpret_cast<uint64_t*>(s.vnew + ATT_D);
  s.flag = flag;
  return s;
}
// The barriers of a unit's tile buffers: one arrival per lane of the warp.
constexpr int ATT_BAR_COUNT = 32;

// Barrier over the unit's 128 threads (barrier 0 when the unit is the whole CTA).
__device__ __forceinline__ void att_sync(int bar) { named_bar_sync(bar, ATT_THREADS); }

// K / V tile layout in shared memory: row r (a key) is 256 bytes; its 16-byte
// chunk c (8 dimensions) sits at chunk position c ^ (r & 7), so the 8 rows an
// ldmatrix reads at one chunk fall in 8 different bank groups.
__device__ __forceinline__ uint32_t att_swz(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D = A (16x16 bf16, row) x B (16x8 bf16, col) + D, fp32 accumulate.  A rows
// 8..15 are zero here (at most 8 query heads), so only a0 / a2 are passed.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16_16816_full(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                    uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

// One unit on threads t = 0..127 of the caller, synchronised by barrier `bar`.
// Warp w takes the tiles w, w + 4, w + 8, ... of the unit's range, two in
// flight, with an online softmax over them.  Both products run on the tensor
// cores (mma.sync m16n8k16, bf16 in, fp32 accumulate):
//   S^T [heads x keys] = Q K^T   (A = queries, rows 0..G-1 of 16; B = K rows)
//   O^T [dims x heads] += V^T P^T (A = V tile, transposed by ldmatrix; B = the
//                                  probabilities, taken straight from the S^T
//                                  fragments as a bf16 pair hi + lo, so P keeps
//                                  16 significant bits: two MMAs per tile row;
//                                  hi and lo each one paired conversion)
// The softmax runs in base 2: the scores carry scale * log2 e, and every
// exponential (tile, rescale, and the merges of warps and of context parts)
// is exp2f of a difference of such scores.  On B200 this took config 4's
// attention from 45.2 / 71.8 to 43.9 / 69.4 us per launch at 32 / 64
// sequences and the config 2 step from 1468 to 1455 us.
// The mbarriers in `sm.bars` are initialised (count ATT_BAR_COUNT) by the
// caller; `tiles_done` counts the tiles this warp consumed before (warp-
// uniform, kept by the caller across units), which fixes buffer and parity.
// Returns false after a timed-out copy (the device status holds the error).
template <int G>
__device__ __forceinline__ bool attn_unit(const AttnParams& p, int b, int g, int sp, const AttnSmem& sm,
                                          uint32_t& tiles_done, int t, int bar) {
  static_assert(G >= 1 && G <= 8, "at most 8 query heads per KV head");
  const int lane = t & 31, warp = t >> 5;
  const int pos = p.positions[b];
  if (pos < 0 || pos >= p.max_len || pos >= p.rope_len || pos >= p.max_ctx) {
    if (t == 0 && sp == 0) record_error(DEV_ERR_BOUNDS, 300);
    return true;
  }
  const int L = pos + 1;
  int nparts = 1, span = L;  // one unit per (b, g): no divides before the first copies
  if (p.nsplit > 1) att_parts(L, p.nsplit, p.max_ctx, nparts, span);
  if (sp >= nparts) return true;
  const int r0 = sp * span, r1 = min(L, r0 + span);
  const int ntiles = (r1 - r0 + ATT_TILE - 1) / ATT_TILE;
  const int ntw = ntiles > warp ? (ntiles - warp + ATT_WARPS - 1) / ATT_WARPS : 0;  // tiles of this warp

  const size_t cache_row0 = ((size_t)b * p.n_kv + g) * p.max_len;
  uint16_t* kc = p.k_cache + cache_row0 * ATT_D;
  uint16_t* vc = p.v_cache + cache_row0 * ATT_D;
  const uint32_t td0 = tiles_done;
  auto tile_t0 = [&](int i) { return r0 + (warp + i * ATT_WARPS) * ATT_TILE; };
  auto tile_buf = [&](int i) {
    return sm.tiles + (size_t)(warp * ATT_NBUF + ((td0 + i) & 1)) * 2 * ATT_TILE_BYTES;
  };
  auto tile_bar = [&](int i) { return &sm.bars[warp * ATT_NBUF + ((td0 + i) & 1)]; };
  auto tile_parity = [&](int i) { return (uint32_t)(((td0 + i) >> 1) & 1); };
  // Every lane copies 16 of the tile's 512 16-byte chunks (K then V, 16 per
  // row) into the swizzled layout; rows past the range are zero-filled.
  auto issue = [&](int i) {
    const int t0 = tile_t0(i), nk = min(ATT_TILE, r1 - t0);
    const uint32_t base = smem_u32(tile_buf(i));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int q = lane + 32 * k;
      const int tensor = q >> 8, row = (q >> 4) & 15, c = q & 15;
      const bool in = row < nk;
      const uint16_t* src = (tensor ? vc : kc) + (size_t)(t0 + (in ? row : 0)) * ATT_D + c * 8;
      cp_async16_zfill(base + tensor * ATT_TILE_BYTES + att_swz(row, c), src, in ? 16u : 0u);
    }
    cp_async_arrive_noinc(tile_bar(i));
  };
  for (int i = 0; i < min(ntw, ATT_NBUF); ++i) issue(i);

  // ---- 1. RoPE on the G query heads and the new key; stage the new value ----
  const int row_elems = (p.n_heads + 2 * p.n_kv) * ATT_D;
  const uint16_t* qkv = p.qkv + (size_t)b * row_elems;
  if (t < ATT_D / 2) {
    const int i = t;
    const float c = bf16_bits_to_f32(p.rope_cos[(size_t)pos * (ATT_D / 2) + i]);
    const float s = bf16_bits_to_f32(p.rope_sin[(size_t)pos * (ATT_D / 2) + i]);
#pragma unroll
    for (int hh = 0; hh <= G; ++hh) {
      const uint16_t* src = (hh < G) ? qkv + (size_t)(g * G + hh) * ATT_D : qkv + (size_t)(p.n_heads + g) * ATT_D;
      const float x1 = bf16_bits_to_f32(src[i]);
      const float x2 = bf16_bits_to_f32(src[i + 64]);
      const float o1 = round_bf16(__fadd_rn(round_bf16(__fmul_rn(x1, c)), round_bf16(__fmul_rn(-x2, s))));
      const float o2 = round_bf16(__fadd_rn(round_bf16(__fmul_rn(x2, c)), round_bf16(__fmul_rn(x1, s))));
      uint16_t* dst = (hh < G) ? sm.qb + hh * ATT_QROW : sm.knew;
      dst[i] = f32_to_bf16_bits(o1);
      dst[i + 64] = f32_to_bf16_bits(o2);
    }
  } else {
    const int i = t - ATT_D / 2;  // 64 threads x 2 values
    reinterpret_cast<uint32_t*>(sm.vnew)[i] =
        reinterpret_cast<const uint32_t*>(qkv + (size_t)(p.n_heads + p.n_kv + g) * ATT_D)[i];
  }
  att_sync(bar);
  if (sp == nparts - 1 && t < 32) {  // append row `pos` (16 B per lane: 16 lanes K, 16 lanes V)
    const int part = t >> 4, c = t & 15;
    uint16_t* dst = (part == 0 ? kc : vc) + (size_t)pos * ATT_D;
    const uint16_t* src = part == 0 ? sm.knew : sm.vnew;
    reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
  }

  // ---- 2. this warp's tiles, online softmax ----
  // query fragments (A operand rows = heads): dims 16 ks + 2 (lane % 4) and + 8
  const int qr = lane >> 2, qc = 2 * (lane & 3);
  uint32_t qa0[8], qa2[8];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qa0[ks] = qr < G ? *reinterpret_cast<const uint32_t*>(sm.qb + qr * ATT_QROW + 16 * ks + qc) : 0u;
    qa2[ks] = qr < G ? *reinterpret_cast<const uint32_t*>(sm.qb + qr * ATT_QROW + 16 * ks + 8 + qc) : 0u;
  }
  float m_run = -INFINITY, l_run = 0.f;  // softmax state of head qr (lanes 4 qr .. 4 qr + 3)
  // O^T fragments: m-tile mt holds dims 16 mt + qr (e 0, 1) and + 8 (e 2, 3),
  // heads qc (e 0, 2) and qc + 1 (e 1, 3)
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
  // ldmatrix row addresses: lane -> matrix lane / 8, row lane % 8
  const int mi = lane >> 3, mr = lane & 7;
  int done = 0;
  bool ok = true;
  for (int i = 0; i < ntw; ++i) {
    const int t0 = tile_t0(i), nk = min(ATT_TILE, r1 - t0);
    uint8_t* buf = tile_buf(i);
    ok = __all_sync(0xffffffffu, mbar_wait(tile_bar(i), tile_parity(i), 301));
    if (!ok) break;
    if (pos >= t0 && pos < t0 + nk) {  // the new row: from shared memory
      const int r = pos - t0, c = lane & 15;
      const uint16_t* src = lane < 16 ? sm.knew : sm.vnew;
      *reinterpret_cast<uint4*>(buf + (lane >> 4) * ATT_TILE_BYTES + att_swz(r, c)) =
          reinterpret_cast<const uint4*>(src)[c];
      __syncwarp();
    }
    const uint32_t kb = smem_u32(buf), vb = kb + ATT_TILE_BYTES;
    // S^T [heads x keys]: two n-tiles of 8 keys
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // matrices: (keys 0-7, chunk 2ks), (keys 0-7, 2ks+1), (keys 8-15, 2ks), (keys 8-15, 2ks+1)
      const int key = (mi >> 1) * 8 + mr;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kb + att_swz(key, 2 * ks + (mi & 1)), b0, b1, b2, b3);
      mma_bf16_16816(s0, qa0[ks], qa2[ks], b0, b1);
      mma_bf16_16816(s1, qa0[ks], qa2[ks], b2, b3);
    }
    // row qr, keys qc, qc+1, 8+qc, 8+qc+1
    float sv[4] = {s0[0], s0[1], s1[0], s1[1]};
    const int kk[4] = {qc, qc + 1, 8 + qc, 9 + qc};
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sv[e] = kk[e] < nk ? sv[e] * (p.scale * 1.4426950408889634f) : -INFINITY;
      mx = fmaxf(mx, sv[e]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float corr = exp2f(m_run - m_new);  // exp(-inf) = 0 on the first tile
    float ev[4], es = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ev[e] = kk[e] < nk ? exp2f(sv[e] - m_new) : 0.f;
      es += ev[e];
    }
    es += __shfl_xor_sync(0xffffffffu, es, 1);
    es += __shfl_xor_sync(0xffffffffu, es, 2);
    l_run = l_run * corr + es;
    m_run = m_new;
    // rescale: this lane's accumulators belong to heads qc and qc + 1, whose
    // state lives in lanes 4 qc and 4 qc + 4
    const float c_lo = __shfl_sync(0xffffffffu, corr, 4 * qc);
    const float c_hi = __shfl_sync(0xffffffffu, corr, (4 * qc + 4) & 31);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[j][0] *= c_lo;
      acc[j][1] *= c_hi;
      acc[j][2] *= c_lo;
      acc[j][3] *= c_hi;
    }
    // P^T (B operand, k = keys, n = heads) straight from the score fragments,
    // split into bf16 hi + lo parts (the products with bf16 V are exact in fp32)
    uint32_t pbw[2], plw[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const __nv_bfloat162 hv = __floats2bfloat162_rn(ev[2 * e], ev[2 * e + 1]);
      pbw[e] = *reinterpret_cast<const uint32_t*>(&hv);
      const __nv_bfloat162 lv = __floats2bfloat162_rn(__fsub_rn(ev[2 * e], __uint_as_float(pbw[e] << 16)),
                                                      __fsub_rn(ev[2 * e + 1], __uint_as_float(pbw[e] & 0xFFFF0000u)));
      plw[e] = *reinterpret_cast<const uint32_t*>(&lv);
    }
    const uint32_t pb0 = pbw[0], pb1 = pbw[1], pl0 = plw[0], pl1 = plw[1];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      // matrices (transposed): (keys 0-7, chunk 2mt), (keys 0-7, 2mt+1), (keys 8-15, 2mt), (keys 8-15, 2mt+1)
      const int key = (mi >> 1) * 8 + mr;
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vb + att_swz(key, 2 * mt + (mi & 1)), a0, a1, a2, a3);
      mma_bf16_16816_full(acc[mt], a0, a1, a2, a3, pb0, pb1);
      mma_bf16_16816_full(acc[mt], a0, a1, a2, a3, pl0, pl1);
    }
    // Reuse the buffer: every lane is done reading it before the next copies.
    __syncwarp();
    done = i + 1;
    if (i + ATT_NBUF < ntw) issue(i + ATT_NBUF);
  }
  // Copies still in flight after a time-out land before the buffers are reused.
  for (int i = done; i < min(ntw, done + ATT_NBUF); ++i) mbar_wait(tile_bar(i), tile_parity(i), 302);
  tiles_done = td0 + (uint32_t)ntw;
  if (!ok && lane == 0) *sm.flag = -1;
  att_sync(bar);
  if (*sm.flag == -1) return false;

  // ---- 3. merge the warp states (tile buffers are free now) ----
  float* sm_m = reinterpret_cast<float*>(sm.tiles);  // [warp][G]
  float* sm_l = sm_m + ATT_WARPS * G;                // [warp][G]
  float* sm_acc = sm_l + ATT_WARPS * G;              // [warp][G][128]
  if (qr < G && (lane & 3) == 0) {
    sm_m[warp * G + qr] = m_run;
    sm_l[warp * G + qr] = l_run;
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d = 16 * mt + qr;
    if (qc < G) {
      sm_acc[(warp * G + qc) * ATT_D + d] = acc[mt][0];
      sm_acc[(warp * G + qc) * ATT_D + d + 8] = acc[mt][2];
    }
    if (qc + 1 < G) {
      sm_acc[(warp * G + qc + 1) * ATT_D + d] = acc[mt][1];
      sm_acc[(warp * G + qc + 1) * ATT_D + d + 8] = acc[mt][3];
    }
  }
  att_sync(bar);
  uint16_t* out_b = p.out + (size_t)b * p.n_heads * ATT_D + (size_t)g * G * ATT_D;
  const size_t pf = (size_t)att_part_floats(G);
  float* part_base = p.ws_part + ((size_t)b * p.n_kv + g) * p.nsplit * pf;
  for (int idx = t; idx < G * ATT_D; idx += ATT_THREADS) {
    const int hh = idx / ATT_D, d = idx % ATT_D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, sm_m[w * G + hh]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) {
      const float f = (sm_l[w * G + hh] > 0.f) ? exp2f(sm_m[w * G + hh] - M) : 0.f;
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
  if (nparts == 1) {
    att_sync(bar);  // shared memory is reused by the group's next unit
    return true;
  }

  // ---- 4. the last unit of (b, g) merges the parts ----
  __threadfence();
  att_sync(bar);
  if (t == 0) {
    int* cnt = p.ws_count + (size_t)b * p.n_kv + g;
    const int old = atomicAdd(cnt, 1);
    const int last = (old == nparts - 1);
    if (last) atomicExch(cnt, 0);  // ready for the next launch
    *sm.flag = last;
  }
  att_sync(bar);
  const bool last = *sm.flag == 1;
  if (last) {
    __threadfence();
    for (int idx = t; idx < G * ATT_D; idx += ATT_THREADS) {
      const int hh = idx / ATT_D;
      float M = -INFINITY;
      for (int s = 0; s < nparts; ++s) M = fmaxf(M, __ldcg(part_base + s * pf + hh));
      float num = 0.f, den = 0.f;
      for (int s = 0; s < nparts; ++s) {
        const float* part = part_base + s * pf;
        const float ls = __ldcg(part + G + hh);
        const float f = (ls > 0.f) ? exp2f(__ldcg(part + hh) - M) : 0.f;
        num = fmaf(__ldcg(part + 2 * G + idx), f, num);
        den = fmaf(ls, f, den);
      }
      out_b[idx] = f32_to_bf16_bits(num / den);
    }
  }
  att_sync(bar);
  if (t == 0) *sm.flag = 0;
  return true;
}

// Standalone launch: grid (B, n_kv_heads, nsplit), one unit per CTA.
template <int G>
__global__ void __launch_bounds__(ATT_THREADS) gqa_decode_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_att[];
  __shared__ int s_flag;
  const AttnSmem sm = att_carve(smem_att, smem_att + ATT_TILES_BYTES, G, &s_flag);
  pdl_trigger();  // the next kernel may launch; it waits for this grid before reading
  const int t = threadIdx.x;
  if (t == 0) {
    for (int i = 0; i < ATT_WARPS * ATT_NBUF; ++i) mbar_init(&sm.bars[i], ATT_BAR_COUNT);
    s_flag = 0;
    fence_mbar_init();
  }
  // The K / V rows below the new position were written by earlier steps and
  // have since left L2 (the step streams over a gigabyte of weights), so the
  // unit asks for its rows while the previous kernel still runs.  A hint only:
  // the position may not be final yet (it is read before griddepcontrol.wait),
  // so it is clamped to the cache and the real loads come after the wait.
  if (t == 0 && p.prefetch) {
    int pos = p.positions[blockIdx.x];
    pos = pos < 0 ? 0 : (pos >= p.max_len ? p.max_len - 1 : pos);
    if (pos >= p.max_ctx) pos = p.max_ctx - 1;
    int nparts = 1, span = pos + 1;
    if (p.nsplit > 1) att_parts(pos + 1, p.nsplit, p.max_ctx, nparts, span);
    const int r0 = (int)blockIdx.z * span, r1 = min(pos, r0 + span);  // row pos is written by this unit
    if (r1 > r0) {
      const size_t row0 = (((size_t)blockIdx.x * p.n_kv + blockIdx.y) * p.max_len + r0) * ATT_D;
      const uint32_t bytes = (uint32_t)(r1 - r0) * ATT_D * 2;
      prefetch_l2_bulk(p.k_cache + row0, bytes);
      prefetch_l2_bulk(p.v_cache + row0, bytes);
    }
  }
  __syncthreads();
  pdl_wait();
  uint32_t tiles_done = 0;
  attn_unit<G>(p, blockIdx.x, blockIdx.y, blockIdx.z, sm, tiles_done, t, 0);
}

}  // namespace bitnet
