// Shared device helpers for the B200 (sm_100a) BitLinear decode path.
//
// Everything here is hand-written inline PTX for the Blackwell execution model:
// mbarriers, bulk (TMA) global->shared copies, tcgen05 tensor-memory allocation,
// tcgen05.mma / commit / ld / st, and programmatic dependent launch (PDL).
//
// Every wait on an mbarrier is bounded by a clock64() budget.  When a wait runs
// out, the kernel records BITNET_DEV_ERR_TIMEOUT in the library's device status
// word (g_bitnet_dev_status) and takes its orderly exit path instead of spinning
// forever; the host reads the word back through bitnet_last_device_status().
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace bitnet {

// ---------------------------------------------------------------------------
// device status word
// ---------------------------------------------------------------------------
enum DevStatus : int {
  DEV_OK = 0,
  DEV_ERR_TIMEOUT = 1,      // an mbarrier wait exceeded its cycle budget
  DEV_ERR_BOUNDS = 2,       // a kernel's own bounds check rejected an index
};

// One word per process and device; written with atomicCAS so the first error wins.
__device__ int g_bitnet_dev_status = 0;
// Where the first timeout happened (kernel-specific site id), for diagnostics.
__device__ int g_bitnet_dev_site = 0;

__device__ __forceinline__ void record_error(int code, int site) {
  if (atomicCAS(&g_bitnet_dev_status, 0, code) == 0) g_bitnet_dev_site = site;
}

// ~2 s at 1.9 GHz.  Real waits in these kernels are microseconds.
constexpr long long kSpinLimitCycles = 4000000000LL;

// ---------------------------------------------------------------------------
// bf16 helpers (explicit IEEE round-to-nearest-even everywhere)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
// Round an fp32 value to the nearest bf16 and return it widened back to fp32.
__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_f32(f32_to_bf16_bits(f));
}

// ---------------------------------------------------------------------------
// shared-memory addressing, mbarriers, bulk copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded busy-poll (non-suspending test_wait) for hand-offs that are expected
// to complete within a microsecond; same contract as mbar_wait.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_test_wait(bar, parity)) {
    if (clock64() - t0 > kSpinLimitCycles) {
      record_error(DEV_ERR_TIMEOUT, site);
      return false;
    }
  }
  return true;
}
// Bounded wait for the phase with the given parity to complete.  Returns false
// (and records the error) when the cycle budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kSpinLimitCycles) {
      record_error(DEV_ERR_TIMEOUT, site);
      return false;
    }
  }
  return true;
}

// Same wait with acquire at cluster scope: for data that other CTAs of the
// cluster store with st.async (whose complete_tx releases at cluster scope).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int site) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > kSpinLimitCycles) {
      record_error(DEV_ERR_TIMEOUT, site);
      return false;
    }
  }
  return true;
}

// Bulk asynchronous copy global -> this CTA's shared memory; completion is
// signalled on `bar` as transaction bytes.  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same, with an L2 evict-first hint: weights are streamed exactly once per step.
__device__ __forceinline__ void bulk_g2s_stream(void* smem_dst, const void* gsrc, uint32_t bytes,
                                                uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Hint: bring [gsrc, gsrc + bytes) into L2 (16-byte aligned, bytes a multiple
// of 16).  No data moves into the CTA and nothing is waited on.
__device__ __forceinline__ void prefetch_l2_bulk(const void* gsrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Barrier among the first `nthreads` threads that use barrier `id` (1..15;
// 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------
// Block until the preceding kernel in the stream (launched with programmatic
// serialisation) has completed and its memory is visible.  No-op otherwise.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to begin its prologue.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// cluster helpers (distributed shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Map a local shared address to the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Non-blocking 4-byte store into a cluster peer's shared memory (addr and mbar
// are shared::cluster addresses of the same CTA, from mapa); the 4 bytes count
// as transaction bytes on that CTA's barrier, whose completion makes them
// visible to its waiters.
__device__ __forceinline__ void st_async_s32(uint32_t addr_cluster, int v, uint32_t mbar_cluster) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.s32 [%0], %1, [%2];" ::"r"(addr_cluster),
               "r"(v), "r"(mbar_cluster)
               : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads and stores
// ---------------------------------------------------------------------------
// Executed by one full warp.  Writes the TMEM base address to *smem_result.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] x B[smem]^T, bf16 x bf16 -> fp32.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor (32-bit) fields, sm_100 UMMA format:
//   [4,6) D format (1 = f32, 2 = s32); [7,10) A format; [10,13) B format;
//   [15] A major (0 = K); [16] B major (0 = K); [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_i8_s32(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor, K-major, no swizzle ("interleaved" core
// matrices of 8 rows x 16 bytes, each core matrix 128 contiguous bytes).
//   lbo: byte distance between core matrices adjacent along K
//   sbo: byte distance between core matrices adjacent along M/N (8-row groups)
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for sm_100
  return d;                 // base offset 0, layout type 0 (no swizzle)
}

// 32 lanes x 32 bits, 16 consecutive columns: each thread writes its own lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 16 consecutive columns into registers.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// 2-bit ternary unpack
// ---------------------------------------------------------------------------
// A 32-bit word of the device weight layout holds 16 ternary codes (code = w + 1
// in {0,1,2}); the code of element e = 4*j + b sits at bits [8*b + 2*j, +2).
// Word j of the output therefore is (x >> 2j) & 0x03030303: four int8 codes for
// four consecutive K positions.
__device__ __forceinline__ void unpack16(uint32_t x, uint32_t& o0, uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  o0 = x & 0x03030303u;
  o1 = (x >> 2) & 0x03030303u;
  o2 = (x >> 4) & 0x03030303u;
  o3 = (x >> 6) & 0x03030303u;
}

// ---------------------------------------------------------------------------
// layouts shared by the kernels and the host
// ---------------------------------------------------------------------------
// Packed weights: [N/128 row blocks][K/64 chunks][128 rows][16 bytes].
__host__ __device__ __forceinline__ size_t wlayout_offset(int n, int kc, int KC) {
  return ((size_t)(n >> 7) * KC + kc) * 2048u + (size_t)(n & 127) * 16u;
}
// Quantised activations: token tiles of T rows; inside a tile
// [K/16 chunks][T/8 row groups][8 rows][16 bytes] (tcgen05 core-matrix order).
__host__ __device__ __forceinline__ size_t alayout_offset(int m, int k, int T, int Kp) {
  const int mt = m / T, mr = m - mt * T;
  return (size_t)mt * T * Kp + ((size_t)(k >> 4) * (T >> 3) + (mr >> 3)) * 128u + (size_t)(mr & 7) * 16u +
         (size_t)(k & 15);
}

// ---------------------------------------------------------------------------
// Pairs of fp32 values in one 64-bit register, for the sm_100 .f32x2
// arithmetic: one instruction performs two IEEE round-to-nearest operations,
// each exactly as its scalar form.  Element 0 sits in the low half.
__device__ __forceinline__ uint64_t f2_make(uint32_t lo_bits, uint32_t hi_bits) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo_bits), "r"(hi_bits));
  return d;
}
__device__ __forceinline__ void f2_split(uint64_t a, uint32_t& lo_bits, uint32_t& hi_bits) {
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo_bits), "=r"(hi_bits) : "l"(a));
}
__device__ __forceinline__ uint64_t f2_splat(float v) { return f2_make(__float_as_uint(v), __float_as_uint(v)); }
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Do not feed an f2_mul result straight into f2_add: on B200 that pair gave
// the rounding of the exact sum (as a fused multiply-add would), not two
// roundings.  Add only operands that went through another rounding step.
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// two packed bf16 values -> an fp32 pair (exact: a bf16 is the top half of an fp32)
__device__ __forceinline__ uint64_t f2_from_bf2(uint32_t v) { return f2_make(v << 16, v & 0xFFFF0000u); }
// fp32 pair -> two bf16 values, each rounded to nearest even, one conversion
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t a) {
  uint32_t lo, hi;
  f2_split(a, lo, hi);
  const __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(lo), __uint_as_float(hi));
  return *reinterpret_cast<const uint32_t*>(&b);
}

}  // namespace bitnet
