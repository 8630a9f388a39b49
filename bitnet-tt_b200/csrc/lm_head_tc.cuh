// lm_head on the tcgen05 tensor cores with the greedy argmax fused into the
// epilogue.
//
// logits[b, v] = bf16(sum_k h[b, k] * W[v, k]) with fp32 accumulation in tensor
// memory; token[b] = argmax_v logits[b, v], smallest index on ties.
//
// Persistent kernel, one CTA per SM, warp-specialised (192 threads):
//   warp 4  producer: streams, for every (vocab tile, 128-wide K stage), the
//           32 KB of the tile's weights and the matching slice of the tiled
//           hidden states into a ring of shared-memory slots (bulk copies,
//           one mbarrier per slot);
//   warp 5  MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> fp32), A = 128
//           vocabulary rows x 16 K, B = T tokens x 16 K, D = 128 x T fp32 in
//           TMEM, double-buffered across tiles so the epilogue of one tile
//           overlaps the MMAs of the next;
//   warps 0-3 epilogue: tcgen05.ld of D (thread = vocabulary row), round to
//           bf16, per-token (max, index) across the tile, running best per
//           token across the CTA's tiles; the CTA's best pairs go to the
//           workspace and argmax_reduce_kernel finishes the job.
#pragma once
#include "common.cuh"
#include "lm_head.cuh"

namespace bitnet {

constexpr int LMT_THREADS = 192;
// 16 x 8 bf16 = 128 K per stage: a stage's weights are one 32 KB bulk copy.
// Measured on B200 (B = 1 and 32): 16 KB copies (8 chunks) reach 4.6-4.9 TB/s,
// 32 KB copies 6.0 TB/s -- an SM's bulk copies carry a large fixed cost each.
constexpr int LMT_STAGE_CHUNKS = 16;
constexpr int LMT_MAX_SLOTS = 12;
constexpr int LMT_PRODUCERS = 4;

struct LmTcParams {
  const uint8_t* w;      // tiled weights [V/128][K/8][128][8 bf16]
  const uint8_t* h;      // tiled hidden [K/8][T/8][8][8 bf16] (T rows, zero padded)
  int B, T, K8, V, ntiles;
  int nslot;
  ArgPair* part;         // [gridDim.x][B]
  uint16_t* logits;      // nullable, [B][V]
};

struct LmTcCtrl {
  uint64_t full[LMT_MAX_SLOTS];
  uint64_t empty[LMT_MAX_SLOTS];
  uint64_t d_full[2];
  uint64_t d_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  float best_v[4][256];
  int best_i[4][256];
};



__host__ __device__ __forceinline__ int lmt_slot_bytes(int T) { return LMT_STAGE_CHUNKS * 2048 + LMT_STAGE_CHUNKS * 16 * T; }
__host__ __device__ __forceinline__ int lmt_ctrl_bytes() { return (int)((sizeof(LmTcCtrl) + 1023) / 1024) * 1024; }

// Rearrange h [B, K] (bf16, row-major) into the tiled B-operand layout with T rows.
__global__ void tile_hidden_kernel(const uint16_t* __restrict__ h, int B, int K, int T, int K8, uint4* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int total = K8 * T;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c = i / T, m = i % T;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < B) {
      const uint16_t* src = h + (size_t)m * K + c * 8;
      if (c * 8 + 8 <= K && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        uint16_t e[8];
        for (int j = 0; j < 8; ++j) e[j] = (c * 8 + j < K) ? src[j] : (uint16_t)0;
        v = make_uint4((uint32_t)e[0] | ((uint32_t)e[1] << 16), (uint32_t)e[2] | ((uint32_t)e[3] << 16),
                       (uint32_t)e[4] | ((uint32_t)e[5] << 16), (uint32_t)e[6] | ((uint32_t)e[7] << 16));
      }
    }
    // core matrix (c, m/8), row m%8
    out[((size_t)c * (T >> 3) + (m >> 3)) * 8 + (m & 7)] = v;
  }
}

__global__ void __launch_bounds__(LMT_THREADS, 1) lm_head_tc_kernel(const LmTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_lmt[];
  LmTcCtrl* ctrl = reinterpret_cast<LmTcCtrl*>(smem_lmt);
  uint8_t* ring = smem_lmt + lmt_ctrl_bytes();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T, K8 = p.K8, nslot = p.nslot;
  const int slot_bytes = lmt_slot_bytes(T);
  const int nstage = (K8 + LMT_STAGE_CHUNKS - 1) / LMT_STAGE_CHUNKS;
  const uint32_t ncols = (2 * T <= 32) ? 32 : (2 * T <= 64 ? 64 : (2 * T <= 128 ? 128 : (2 * T <= 256 ? 256 : 512)));
  volatile int* abort_flag = &ctrl->abort_flag;
  const int my_tiles = (p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < nslot; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctrl->d_full[b], 1);
      mbar_init(&ctrl->d_empty[b], 128);
    }
    ctrl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&ctrl->tmem_base, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tbase = ctrl->tmem_base;

  auto wait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity, site)) {
      *abort_flag = 1;
      return false;
    }
    return true;
  };

  if (warp == 4) {
    // ---------------- producer ----------------
    // Lanes 0..nprod-1 each own the stages it = lane (mod nprod): a thread's
    // bulk copies complete one after another, so a single producer thread
    // cannot keep the ring full.  Each lane waits only on barriers armed by the
    // MMA issuer (another warp), and nprod <= nslot, so a lane never waits for
    // a slot whose previous stage belongs to a lane of the same round.
    const int nprod = min(LMT_PRODUCERS, nslot);
    if (lane < nprod) {
      const uint64_t policy = l2_policy_evict_first();
      const int total = my_tiles * nstage;
      auto stage_of = [&](int it, int& vt, int& c0, int& nch) {
        vt = blockIdx.x + (it / nstage) * gridDim.x;
        c0 = (it % nstage) * LMT_STAGE_CHUNKS;
        nch = min(LMT_STAGE_CHUNKS, K8 - c0);
      };
      // The weights do not depend on the previous kernel: fill the ring's first
      // slots with them before waiting for the tiled hidden states.
      const int pre = min(nslot, total);
      for (int it = lane; it < pre; it += nprod) {
        int vt, c0, nch;
        stage_of(it, vt, c0, nch);
        mbar_arrive_expect_tx(&ctrl->full[it], (uint32_t)(nch * 2048 + nch * 16 * T));
        bulk_g2s_stream(ring + (size_t)it * slot_bytes, p.w + ((size_t)vt * K8 + c0) * 2048, nch * 2048,
                        &ctrl->full[it], policy);
      }
      pdl_wait();
      for (int it = lane; it < pre; it += nprod) {
        int vt, c0, nch;
        stage_of(it, vt, c0, nch);
        bulk_g2s(ring + (size_t)it * slot_bytes + LMT_STAGE_CHUNKS * 2048, p.h + (size_t)c0 * 16 * T, nch * 16 * T,
                 &ctrl->full[it]);
      }
      int issued = -1;  // last stage this lane issued
      if (lane < pre) issued = lane + ((pre - 1 - lane) / nprod) * nprod;
      for (int it = pre + lane; it < total; it += nprod) {
        const int slot = it % nslot;
        if (!wait(&ctrl->empty[slot], ((it / nslot) + 1) & 1, 400)) break;
        int vt, c0, nch;
        stage_of(it, vt, c0, nch);
        uint8_t* dst = ring + (size_t)slot * slot_bytes;
        mbar_arrive_expect_tx(&ctrl->full[slot], (uint32_t)(nch * 2048 + nch * 16 * T));
        bulk_g2s_stream(dst, p.w + ((size_t)vt * K8 + c0) * 2048, nch * 2048, &ctrl->full[slot], policy);
        bulk_g2s(dst + LMT_STAGE_CHUNKS * 2048, p.h + (size_t)c0 * 16 * T, nch * 16 * T, &ctrl->full[slot]);
        issued = it;
      }
      if (*abort_flag) {
        // Let this lane's copies land before the shared memory is released.
        // Older stages of the lane had their slot refilled, so they landed.
        for (int it = max(0, issued - nslot + 1); it <= issued; ++it) {
          const bool mine = (it < pre) ? (it % nprod == lane) : ((it - pre) % nprod == lane);
          if (mine) mbar_wait(&ctrl->full[it % nslot], (it / nslot) & 1, 404);
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, T);
      int it = 0;
      for (int i = 0; i < my_tiles && !*abort_flag; ++i) {
        const int db = i & 1;
        if (i >= 2 && !wait(&ctrl->d_empty[db], ((i >> 1) + 1) & 1, 401)) break;
        tc_fence_after();
        const uint32_t d = tbase + db * T;
        for (int s = 0; s < nstage; ++s, ++it) {
          const int slot = it % nslot;
          if (!wait(&ctrl->full[slot], (it / nslot) & 1, 402)) break;
          tc_fence_after();
          const int nch = min(LMT_STAGE_CHUNKS, K8 - s * LMT_STAGE_CHUNKS);
          const uint32_t a0 = smem_u32(ring + (size_t)slot * slot_bytes);
          const uint32_t b0 = a0 + LMT_STAGE_CHUNKS * 2048;
          for (int kk = 0; kk < nch / 2; ++kk) {  // K = 16 per MMA = 2 chunks
            const uint64_t ad = smem_desc_kmajor(a0 + kk * 4096, 2048, 128);
            const uint64_t bd = smem_desc_kmajor(b0 + kk * 32 * T, 16 * T, 128);
            mma_f16_ss(d, ad, bd, idesc, (s | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&ctrl->empty[slot]);
        }
        tc_commit(&ctrl->d_full[db]);
      }
    }
  } else {
    // ---------------- epilogue (warps 0-3, thread = vocabulary row) ----------------
    for (int b = tid; b < T; b += 128) {
      for (int w = 0; w < 4; ++w) {
        ctrl->best_v[w][b] = -INFINITY;
        ctrl->best_i[w][b] = 0x7fffffff;
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    for (int i = 0; i < my_tiles; ++i) {
      const int db = i & 1;
      if (!wait(&ctrl->d_full[db], (i >> 1) & 1, 403)) break;
      tc_fence_after();
      const int vt = blockIdx.x + i * gridDim.x;
      const int v = vt * 128 + tid;
      const uint32_t tl = tbase + ((uint32_t)(warp * 32) << 16) + db * T;
      for (int c = 0; c < T; c += 16) {
        uint32_t r[16];
        tmem_ld16(tl + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int b = c + j;
          const float lg = round_bf16(__uint_as_float(r[j]));
          if (p.logits != nullptr && b < p.B && v < p.V) p.logits[(size_t)b * p.V + v] = f32_to_bf16_bits(lg);
          float bv = (v < p.V) ? lg : -INFINITY;
          int bi = (v < p.V) ? v : 0x7fffffff;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (arg_better(ov, oi, bv, bi)) {
              bv = ov;
              bi = oi;
            }
          }
          if (lane == 0 && arg_better(bv, bi, ctrl->best_v[warp][b], ctrl->best_i[warp][b])) {
            ctrl->best_v[warp][b] = bv;
            ctrl->best_i[warp][b] = bi;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctrl->d_empty[db]);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    for (int b = tid; b < p.B; b += 128) {
      float bv = ctrl->best_v[0][b];
      int bi = ctrl->best_i[0][b];
      for (int w = 1; w < 4; ++w)
        if (arg_better(ctrl->best_v[w][b], ctrl->best_i[w][b], bv, bi)) {
          bv = ctrl->best_v[w][b];
          bi = ctrl->best_i[w][b];
        }
      p.part[(size_t)blockIdx.x * p.B + b] = ArgPair{bv, bi};
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, ncols);
  }
}

}  // namespace bitnet
