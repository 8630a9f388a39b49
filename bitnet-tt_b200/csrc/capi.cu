// C ABI of the B200 packed-ternary BitLinear decode path (declared in
// include/bitnet_b200.h).  One translation unit: every kernel header is
// included here so the kernels share the device status word.
//
// Host-side responsibilities: argument validation (shapes, alignment, device
// architecture), choice of execution path and K split, and kernel launches
// with programmatic-dependent-launch and cluster attributes.  No entry point
// allocates device memory or synchronises (except bitnet_last_device_status).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>
#include <algorithm>
#include <cmath>

#include "act_quant.cuh"
#include "attention.cuh"
#include "attention_prefill.cuh"
#include "bitlinear_simt.cuh"
#include "bitlinear_tc.cuh"
#include "common.cuh"
#include "decode_layers.cuh"
#include "lm_head.cuh"
#include "lm_head_tc.cuh"
#include "pack.cuh"
#include "../../include/bitnet_b200.h"

using namespace bitnet;

namespace {

constexpr int kAbiVersion = 3;
constexpr int kMaxDevices = 64;
constexpr size_t kMaxDynSmem = 232448;  // 227 KB, the sm_100 per-CTA opt-in limit

std::atomic<int> g_pdl{1};        // programmatic dependent launch on by default
std::atomic<int> g_tc_split{0};   // 0 = automatic K split for the tcgen05 path
std::atomic<int> g_simt_max_m{4}; // AUTO path: SIMT for M <= this

struct DevInfo {
  int checked = 0;  // 0 unknown, 1 ok, -1 unsupported
  int sms = 0;
};
DevInfo g_dev[kMaxDevices];
std::mutex g_mu;

int device_info(DevInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BITNET_ERR_CUDA;
  DevInfo& d = g_dev[dev];
  if (d.checked == 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (d.checked == 0) {
      int major = 0, minor = 0, sms = 0;
      if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return BITNET_ERR_CUDA;
      d.sms = sms;
      d.checked = (major == 10 && minor == 0) ? 1 : -1;
    }
  }
  if (d.checked < 0) return BITNET_ERR_UNSUPPORTED_DEVICE;
  *out = &d;
  return BITNET_OK;
}

thread_local char g_cuda_msg[256] = "no CUDA error recorded";

int cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_cuda_msg, sizeof(g_cuda_msg), "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
  (void)cudaGetLastError();
  return BITNET_ERR_CUDA;
}

int dev_index() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

// Raise the dynamic shared memory limit of a kernel once per device, to the
// per-CTA opt-in limit minus the kernel's static shared memory.
template <typename K>
int ensure_smem(K kernel, std::atomic<unsigned long long>* done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (done_mask->load() & bit) return BITNET_OK;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(kMaxDynSmem - fa.sharedSizeBytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  done_mask->fetch_or(bit);
  return BITNET_OK;
}

template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, bitnet_stream_t stream, int cluster_z,
           Args... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (g_pdl.load()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_z > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = (unsigned)cluster_z;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ((KArgs)args)...);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx");
  return BITNET_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

int act_rows_of(int M) { return M <= 256 ? round_up(M, 16) : round_up(M, 256); }
int act_tile_of(int M) { return M <= 256 ? round_up(M, 16) : 256; }

// One CTA waits on an mbarrier that nothing arrives on; the bounded wait gives
// up after limit_cycles and records the timeout (site 900), then returns.
__global__ void selftest_wait_kernel(long long limit_cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    bool done = mbar_try_wait(&bar, 0);
    while (!done && clock64() - t0 <= limit_cycles) done = mbar_try_wait(&bar, 0);
    if (!done) record_error(DEV_ERR_TIMEOUT, 900);
  }
}

int to_dev_segments(const bitnet_segments_t* s, int N, int epilogue, bitnet_segments_dev* out) {
  memset(out, 0, sizeof(*out));
  if (s == nullptr) {
    out->count = 1;
    out->end[0] = N;
    out->scale[0] = out->scale[1] = 1.0f;
    if (epilogue == BITNET_EPI_RELU2_MUL) out->count = 2;
    return BITNET_OK;
  }
  if (s->count < 1 || s->count > BITNET_MAX_SEGMENTS) return BITNET_ERR_INVALID_ARGUMENT;
  out->count = s->count;
  for (int i = 0; i < s->count; ++i) {
    out->end[i] = s->end[i];
    out->scale[i] = s->scale[i];
  }
  if (epilogue == BITNET_EPI_RELU2_MUL) return s->count == 2 ? BITNET_OK : BITNET_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < s->count; ++i)
    if (s->end[i] <= (i ? s->end[i - 1] : 0)) return BITNET_ERR_INVALID_ARGUMENT;
  return s->end[s->count - 1] == N ? BITNET_OK : BITNET_ERR_INVALID_ARGUMENT;
}

std::atomic<unsigned long long> g_smem_aq{0}, g_smem_aq_stage{0}, g_smem_simt[3][4], g_smem_tc[3], g_smem_lmh{0}, g_smem_att[4],
    g_smem_apf{0};

int lm_head_tile_T(int B) { return round_up(B, 16); }
size_t lm_head_part_bytes(int B, int grid) { return (size_t)grid * B * sizeof(ArgPair); }

template <int EPI, int MT>
int launch_simt(const int8_t* q, const float* rs, const int32_t* rsum, int M, int Kp, int T, const uint8_t* w,
                int N, const bitnet_segments_dev& seg, const uint16_t* res, uint16_t* y, int32_t* acc,
                bitnet_stream_t st, int mt_idx, const SimtFuse& fz) {
  auto k = bitlinear_simt_kernel<EPI, MT>;
  if (int e = ensure_smem(k, &g_smem_simt[EPI][mt_idx])) return e;
  const int rows = 32 * (EPI == EPI_RELU2_MUL ? 2 : 1);
  const size_t smem = (size_t)Kp * 8 + (size_t)8 * MT * 32 * 4;
  if (smem > kMaxDynSmem) return BITNET_ERR_INVALID_ARGUMENT;
  return launch(k, dim3((N + rows - 1) / rows), dim3(SIMT_THREADS), smem, st, 1, q, rs, rsum, M, Kp, T, w, N, seg,
                res, y, acc, fz);
}

template <int EPI>
int dispatch_simt(const int8_t* q, const float* rs, const int32_t* rsum, int M, int Kp, int T, const uint8_t* w,
                  int N, const bitnet_segments_dev& seg, const uint16_t* res, uint16_t* y, int32_t* acc,
                  bitnet_stream_t st, const SimtFuse& fz = SimtFuse{nullptr, 0, 0, nullptr, 0.f}) {
  if (M <= 1) return launch_simt<EPI, 1>(q, rs, rsum, M, Kp, T, w, N, seg, res, y, acc, st, 0, fz);
  if (M <= 2) return launch_simt<EPI, 2>(q, rs, rsum, M, Kp, T, w, N, seg, res, y, acc, st, 1, fz);
  if (M <= 4) return launch_simt<EPI, 4>(q, rs, rsum, M, Kp, T, w, N, seg, res, y, acc, st, 2, fz);
  return launch_simt<EPI, 8>(q, rs, rsum, M, Kp, T, w, N, seg, res, y, acc, st, 3, fz);
}

// Shared-memory request of the tcgen05 BitLinear.  Besides the ring and the
// epilogue buffers it has a floor that caps the number of resident CTAs per SM
// at what tensor memory can serve at once (512 columns per SM): one CTA with
// 512 columns, or two with 256.  Every resident CTA then gets its columns
// immediately, so a CTA of a cluster can never sit in tcgen05.alloc while its
// peers wait for it.
size_t tc_smem_bytes(int T, int nslot, int split, int cols = TC_TMEM_COLS, int sc = TC_STAGE_CHUNKS) {
  const size_t ring = (size_t)nslot * tc_slot_bytes(T, sc);
  const size_t stage = (size_t)T * TC_ST_LD * 2;  // staged bf16 output tile (no K split)
  const size_t recv = (size_t)split * tc_part_bytes(T, split);  // one receive slot per source rank
  size_t bytes = TC_CTRL_BYTES + (split > 1 ? ring + recv : (ring > stage ? ring : stage));
  const size_t floor_bytes = cols == 512 ? (size_t)116 * 1024 : (size_t)77 * 1024;
  return bytes < floor_bytes ? floor_bytes : bytes;
}
size_t tc_smem_limit(int cols) { return cols == 512 ? kMaxDynSmem : (size_t)112 * 1024; }

int tc_nslot(int T, int KC, int split, int cols = TC_TMEM_COLS, int sc = TC_STAGE_CHUNKS) {
  const int chunks_max = (KC + split - 1) / split;
  const int stages_max = (chunks_max + sc - 1) / sc;
  int nslot = TC_MAX_SLOTS;
  if (nslot > stages_max) nslot = stages_max;
  if (nslot < 2) nslot = 2;
  while (nslot > 2 && tc_smem_bytes(T, nslot, split, cols, sc) > tc_smem_limit(cols)) --nslot;
  return nslot;
}

// Clusters of `split` CTAs that can be resident at once (cached per device, T, split, columns).
template <int EPI>
int dispatch_tc(TcParams p, int ntile_n, int ntile_m, bitnet_stream_t st, const DevInfo& dev) {
  auto k = bitlinear_tc_kernel<EPI>;
  if (!(g_smem_tc[EPI].load() & 1ull << (dev_index() & 63))) {
    // all of the SM's unified L1/shared storage as shared memory, so that two
    // 256-column CTAs fit on an SM (also what the occupancy queries assume)
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(carveout)");
  }
  if (int e = ensure_smem(k, &g_smem_tc[EPI])) return e;
  const int tiles = ntile_n * ntile_m;
  int split = g_tc_split.load();
  if (split <= 0) {
    // About 1.25 CTAs per SM: a K split cuts each CTA's chain of MMA stages,
    // and two CTAs share an SM (256 tensor-memory columns each) when there are
    // more CTAs than SMs.  Measured on B200 at 32 tokens: qkv 30 tiles -> 6,
    // o_proj / down 20 tiles -> 8 (4, 6 and 8 tried at the whole-step level).
    split = 1;
    if (ntile_m == 1 && p.T <= 64) {
      split = (5 * dev.sms / 4 + tiles / 2) / tiles;
      const int by_k = p.KC / 4;  // at least one full 256-wide stage per CTA
      if (split > by_k) split = by_k;
      if (split > 8) split = 8;
      if (split < 1) split = 1;
      // With >= 0.7 CTAs per SM already, no split: each CTA's whole K range then
      // sits in its ring, fetched before griddepcontrol.wait, and the partial-sum
      // exchange disappears.  Measured at 32 tokens: gate_up (108 tiles) alone
      // 10.0 -> 11.1 us, but the decode step 17,290 -> 17,440 tok/s, because the
      // weight fetch overlaps the preceding act-quant launch.
      if (tiles * 10 >= dev.sms * 7) split = 1;
    }
  }
  // K chunks per stage.  Halving the stage for 256-token tiles (twice the
  // stages in flight) was measured slower: a stage's copies cost ~0.7 us of
  // fixed time whatever their size, so fewer, larger stages win.  At decode
  // (T <= 64) each stage also costs the MMA issuers ~0.7 us of barrier waits
  // and fences whatever its size (measured on B200 with per-stage timestamps),
  // so the CTA's K range is cut into as few stages of at most
  // TC_MAX_STAGE_CHUNKS chunks as possible, balanced, that still leave an A
  // buffer per stage (up to two) in the tensor memory of the CTAs-per-SM the
  // grid needs.
  int sc = TC_STAGE_CHUNKS;
  const int chunks_max = (p.KC + split - 1) / split;
  if (p.T <= 64) {
    const bool two_per_sm = (long)tiles * split > dev.sms;
    for (int nst = (chunks_max + TC_MAX_STAGE_CHUNKS - 1) / TC_MAX_STAGE_CHUNKS; nst <= chunks_max; ++nst) {
      sc = (chunks_max + nst - 1) / nst;
      const int stages = (chunks_max + sc - 1) / sc;
      if (tc_nbuf(p.T, two_per_sm ? 256 : TC_TMEM_COLS, sc) >= std::min(2, stages)) break;
    }
  }
  const int stages_max = (chunks_max + sc - 1) / sc;
  int cols = TC_TMEM_COLS;
  // two CTAs per SM, when both the tensor memory and the shared memory of the
  // smallest ring fit twice (with an A buffer per stage, up to two)
  if ((long)tiles * split > dev.sms && tc_nbuf(p.T, 256, sc) >= std::min(2, stages_max) &&
      tc_smem_bytes(p.T, 2, split, 256, sc) <= tc_smem_limit(256))
    cols = 256;
  if (split > 8 || split > p.KC) return BITNET_ERR_INVALID_ARGUMENT;
  if (split > 1 && p.T > 64) return BITNET_ERR_INVALID_ARGUMENT;
  const int nslot = tc_nslot(p.T, p.KC, split, cols, sc);
  const size_t smem = tc_smem_bytes(p.T, nslot, split, cols, sc);
  if (smem > tc_smem_limit(cols)) return BITNET_ERR_INVALID_ARGUMENT;
  p.nslot = nslot;
  p.split = split;
  p.tmem_cols = cols;
  p.nbuf = tc_nbuf(p.T, cols, sc);
  p.sc = sc;
  return launch(k, dim3(ntile_n, ntile_m, split), dim3(TC_THREADS), smem, st, split, p);
}

}  // namespace

extern "C" {

int bitnet_abi_version(void) { return kAbiVersion; }


const char* bitnet_last_cuda_error(void) { return g_cuda_msg; }

const char* bitnet_status_string(int status) {
  switch (status) {
    case BITNET_OK: return "ok";
    case BITNET_ERR_INVALID_ARGUMENT: return "invalid argument (shape, null pointer or option out of range)";
    case BITNET_ERR_ALIGNMENT: return "pointer not aligned as required";
    case BITNET_ERR_UNSUPPORTED_DEVICE: return "current CUDA device is not an sm_100 (B200) GPU";
    case BITNET_ERR_CUDA: return "CUDA runtime call failed";
    case BITNET_ERR_DEVICE_TIMEOUT: return "a kernel gave up a bounded wait on the device";
    case BITNET_ERR_SCRATCH_LIMIT:
      return "problem exceeds the static scratch of bitnet_bitlinear_noalloc (see BITNET_NOALLOC_MAX_*)";
    default: return "unknown status";
  }
}

int bitnet_last_device_status(int* site) {
  if (cudaDeviceSynchronize() != cudaSuccess) return BITNET_ERR_CUDA;
  int st = 0, where = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&st, g_bitnet_dev_status, sizeof(int)) != cudaSuccess) return BITNET_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&where, g_bitnet_dev_site, sizeof(int)) != cudaSuccess) return BITNET_ERR_CUDA;
  if (st != 0) {
    cudaMemcpyToSymbol(g_bitnet_dev_status, &zero, sizeof(int));
    cudaMemcpyToSymbol(g_bitnet_dev_site, &zero, sizeof(int));
  }
  if (site) *site = where;
  if (st == DEV_ERR_TIMEOUT) return BITNET_ERR_DEVICE_TIMEOUT;
  if (st == DEV_ERR_BOUNDS) return BITNET_ERR_INVALID_ARGUMENT;
  return BITNET_OK;
}

int bitnet_selftest_bounded_wait(long long limit_cycles, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (limit_cycles < 1 || limit_cycles > (1LL << 31)) return BITNET_ERR_INVALID_ARGUMENT;
  return launch(selftest_wait_kernel, dim3(1), dim3(32), 0, stream, 1, limit_cycles);
}

int bitnet_set_pdl(int enable) {
  g_pdl.store(enable ? 1 : 0);
  return BITNET_OK;
}
int bitnet_set_tc_split(int split) {
  if (split < 0 || split > 8) return BITNET_ERR_INVALID_ARGUMENT;
  g_tc_split.store(split);
  return BITNET_OK;
}
int bitnet_set_simt_max_m(int m) {
  if (m < 0 || m > SIMT_MAX_M) return BITNET_ERR_INVALID_ARGUMENT;
  g_simt_max_m.store(m);
  return BITNET_OK;
}

size_t bitnet_packed_weight_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  return (size_t)round_up(N, 128) * (size_t)(round_up(K, 64) / 4);
}
size_t bitnet_act_bytes(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  return (size_t)act_rows_of(M) * (size_t)round_up(K, 64);
}
int bitnet_act_rows(int M) { return M <= 0 ? 0 : act_rows_of(M); }

static int grid_for(size_t work, int threads) {
  size_t g = (work + threads - 1) / threads;
  if (g > 65535u * 4u) g = 65535u * 4u;
  return (int)(g == 0 ? 1 : g);
}

int bitnet_pack_ternary(const int8_t* w_q, int N, int K, uint8_t* w_packed, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!w_q || !w_packed || N <= 0 || K <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(w_packed, 16)) return BITNET_ERR_ALIGNMENT;
  const int Npad = round_up(N, 128), KC = round_up(K, 64) / 64;
  const size_t words = (size_t)Npad * KC * 4;
  pack_ternary_kernel<<<grid_for(words, 256), 256, 0, (cudaStream_t)stream>>>(w_q, N, K, Npad, KC,
                                                                              reinterpret_cast<uint32_t*>(w_packed));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BITNET_OK : cuda_fail(e, "kernel launch");
}

int bitnet_pack_from_canonical(const uint8_t* canonical, int N, int K, uint8_t* w_packed, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!canonical || !w_packed || N <= 0 || K <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(w_packed, 16)) return BITNET_ERR_ALIGNMENT;
  const int Npad = round_up(N, 128), KC = round_up(K, 64) / 64;
  const size_t words = (size_t)Npad * KC * 4;
  pack_from_canonical_kernel<<<grid_for(words, 256), 256, 0, (cudaStream_t)stream>>>(
      canonical, N, K, Npad, KC, reinterpret_cast<uint32_t*>(w_packed));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BITNET_OK : cuda_fail(e, "kernel launch");
}

size_t bitnet_tilized_weight_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  return (size_t)((K + 31) / 32) * (size_t)((N + 31) / 32) * 256u;
}

int bitnet_pack_from_tilized(const uint8_t* tiles, int N, int K, uint8_t* w_packed, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!tiles || !w_packed || N <= 0 || K <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(w_packed, 16)) return BITNET_ERR_ALIGNMENT;
  const int Npad = round_up(N, 128), KC = round_up(K, 64) / 64;
  const size_t words = (size_t)Npad * KC * 4;
  pack_from_tilized_kernel<<<grid_for(words, 256), 256, 0, (cudaStream_t)stream>>>(
      tiles, N, K, Npad, KC, reinterpret_cast<uint32_t*>(w_packed));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BITNET_OK : cuda_fail(e, "kernel launch");
}

int bitnet_act_quant(const void* x, int M, int K, int ldx, const void* gamma, float eps, int8_t* q, float* row_scale,
                     int32_t* row_sum, void* normed_out, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!x || M <= 0 || K <= 0 || ldx < K) return BITNET_ERR_INVALID_ARGUMENT;
  const bool want_q = q || row_scale || row_sum;
  if (want_q && (!q || !row_scale || !row_sum)) return BITNET_ERR_INVALID_ARGUMENT;
  if (!want_q && !normed_out) return BITNET_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 2) || (gamma && !aligned(gamma, 2)) || (normed_out && !aligned(normed_out, 2)))
    return BITNET_ERR_ALIGNMENT;
  if (q && !aligned(q, 16)) return BITNET_ERR_ALIGNMENT;
  const int Kp = round_up(K, 64);
  const int rows = want_q ? act_rows_of(M) : M;
  const bool vec_ok = K % 8 == 0 && ldx % 8 == 0 && aligned(x, 16) && (!gamma || aligned(gamma, 16)) &&
                      (!normed_out || aligned(normed_out, 16));
  // many rows: a warp per row, rows staged in shared memory (the rows are padded to whole token tiles,
  // multiples of 8)
  if (vec_ok && M >= 256 && rows % 8 == 0 && K <= AQ_STAGE_MAX_K) {
    if (int e = ensure_smem(act_quant_rows_kernel, &g_smem_aq_stage)) return e;
    return launch(act_quant_rows_kernel, dim3(rows / 8), dim3(256), (size_t)16 * K, stream, 1,
                  (const uint16_t*)x, M, K, ldx, (const uint16_t*)gamma, eps, q, row_scale, row_sum,
                  (uint16_t*)normed_out, act_tile_of(M), Kp);
  }
  // few rows: one CTA per row, one thread per chunk of 8 (two or four chunks
  // per thread for rows longer than 8192)
  if (vec_ok && Kp / 8 <= 4 * 1024) {
    const int chunks = Kp / 8;
    const int C = chunks <= 1024 ? 1 : (chunks <= 2048 ? 2 : 4);
    const int threads = ((chunks + C - 1) / C + 31) / 32 * 32;
    auto k = C == 1 ? act_quant_row_kernel<1> : (C == 2 ? act_quant_row_kernel<2> : act_quant_row_kernel<4>);
    return launch(k, dim3(rows), dim3(threads), 0, stream, 1, (const uint16_t*)x, M, K, ldx, (const uint16_t*)gamma,
                  eps, q, row_scale, row_sum, (uint16_t*)normed_out, act_tile_of(M), Kp);
  }
  if (vec_ok && Kp <= 8 * AQ_THREADS * AQ_MAXC)
    return launch(act_quant_vec_kernel, dim3(rows), dim3(AQ_THREADS), 0, stream, 1, (const uint16_t*)x, M, K, ldx,
                  (const uint16_t*)gamma, eps, q, row_scale, row_sum, (uint16_t*)normed_out, act_tile_of(M), Kp);
  const size_t smem = (size_t)Kp * 4;
  if (smem > kMaxDynSmem) return BITNET_ERR_INVALID_ARGUMENT;
  if (int e = ensure_smem(act_quant_kernel, &g_smem_aq)) return e;
  return launch(act_quant_kernel, dim3(rows), dim3(256), smem, stream, 1, (const uint16_t*)x, M, K, ldx,
                (const uint16_t*)gamma, eps, q, row_scale, row_sum, (uint16_t*)normed_out, act_tile_of(M), Kp);
}

int bitnet_bitlinear_q(const int8_t* q, const float* row_scale, const int32_t* row_sum, int M, int K,
                       const uint8_t* w_packed, int N, const bitnet_segments_t* segments, int epilogue,
                       const void* residual, void* y, int32_t* acc_out, int path, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!q || !row_scale || !row_sum || !w_packed || !y || M <= 0 || K <= 0 || N <= 0)
    return BITNET_ERR_INVALID_ARGUMENT;
  if (epilogue < BITNET_EPI_NONE || epilogue > BITNET_EPI_RESIDUAL_ADD) return BITNET_ERR_INVALID_ARGUMENT;
  if (epilogue == BITNET_EPI_RESIDUAL_ADD && !residual) return BITNET_ERR_INVALID_ARGUMENT;
  if (epilogue == BITNET_EPI_RELU2_MUL && (N % 64) != 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(q, 16) || !aligned(w_packed, 16) || !aligned(row_scale, 4) || !aligned(row_sum, 4) ||
      !aligned(y, 2) || (residual && !aligned(residual, 2)) || (acc_out && !aligned(acc_out, 4)))
    return BITNET_ERR_ALIGNMENT;
  bitnet_segments_dev seg;
  if (int e = to_dev_segments(segments, N, epilogue, &seg)) return e;
  const int Kp = round_up(K, 64), T = act_tile_of(M);
  if (path == BITNET_PATH_AUTO) path = (M <= g_simt_max_m.load()) ? BITNET_PATH_SIMT : BITNET_PATH_TCGEN05;
  const uint16_t* res = (const uint16_t*)residual;
  uint16_t* yy = (uint16_t*)y;
  if (path == BITNET_PATH_SIMT) {
    if (M > SIMT_MAX_M) return BITNET_ERR_INVALID_ARGUMENT;
    switch (epilogue) {
      case BITNET_EPI_NONE: return dispatch_simt<EPI_NONE>(q, row_scale, row_sum, M, Kp, T, w_packed, N, seg, res, yy, acc_out, stream);
      case BITNET_EPI_RELU2_MUL: return dispatch_simt<EPI_RELU2_MUL>(q, row_scale, row_sum, M, Kp, T, w_packed, N, seg, res, yy, acc_out, stream);
      default: return dispatch_simt<EPI_RESIDUAL_ADD>(q, row_scale, row_sum, M, Kp, T, w_packed, N, seg, res, yy, acc_out, stream);
    }
  }
  if (path != BITNET_PATH_TCGEN05) return BITNET_ERR_INVALID_ARGUMENT;
  TcParams p;
  memset(&p, 0, sizeof(p));
  p.q = q;
  p.row_scale = row_scale;
  p.row_sum = row_sum;
  p.M = M;
  p.Kp = Kp;
  p.T = T;
  p.w = w_packed;
  p.N = N;
  p.KC = Kp / 64;
  p.seg = seg;
  p.residual = res;
  p.y = yy;
  p.acc_out = acc_out;
  const int ntile_n = round_up(N, 128) / 128, ntile_m = act_rows_of(M) / T;
  switch (epilogue) {
    case BITNET_EPI_NONE: return dispatch_tc<EPI_NONE>(p, ntile_n, ntile_m, stream, *d);
    case BITNET_EPI_RELU2_MUL: return dispatch_tc<EPI_RELU2_MUL>(p, ntile_n, ntile_m, stream, *d);
    default: return dispatch_tc<EPI_RESIDUAL_ADD>(p, ntile_n, ntile_m, stream, *d);
  }
}

int bitnet_bitlinear(const void* x, int M, int K, const void* gamma, float eps, const uint8_t* w_packed, int N,
                     const bitnet_segments_t* segments, int epilogue, const void* residual, void* y, int32_t* acc_out,
                     int8_t* q_ws, float* scale_ws, int32_t* sum_ws, int path, bitnet_stream_t stream) {
  if (!q_ws || !scale_ws || !sum_ws) return BITNET_ERR_INVALID_ARGUMENT;
  // Below the ridge (the CUDA-core path) one launch does everything: each CTA
  // normalises and quantises the few token rows itself (same codes as
  // bitnet_act_quant), so no act-quant launch and no code buffer round trip.
  const int path_r = path == BITNET_PATH_AUTO ? ((M <= g_simt_max_m.load()) ? BITNET_PATH_SIMT : BITNET_PATH_TCGEN05)
                                              : path;
  const int Kp = round_up(K, 64);
  if (path_r == BITNET_PATH_SIMT && x && M > 0 && M <= SIMT_MAX_M && K > 0 && K % 8 == 0 &&
      Kp <= 8 * AQ_THREADS * AQ_MAXC && aligned(x, 16) && (!gamma || aligned(gamma, 16)) && eps >= 0.f) {
    DevInfo* d;
    if (int e = device_info(&d)) return e;
    if (!w_packed || !y || N <= 0) return BITNET_ERR_INVALID_ARGUMENT;
    if (epilogue < BITNET_EPI_NONE || epilogue > BITNET_EPI_RESIDUAL_ADD) return BITNET_ERR_INVALID_ARGUMENT;
    if (epilogue == BITNET_EPI_RESIDUAL_ADD && !residual) return BITNET_ERR_INVALID_ARGUMENT;
    if (epilogue == BITNET_EPI_RELU2_MUL && (N % 64) != 0) return BITNET_ERR_INVALID_ARGUMENT;
    if (!aligned(w_packed, 16) || !aligned(y, 2) || (residual && !aligned(residual, 2)) || (acc_out && !aligned(acc_out, 4)))
      return BITNET_ERR_ALIGNMENT;
    bitnet_segments_dev seg;
    if (int e = to_dev_segments(segments, N, epilogue, &seg)) return e;
    const SimtFuse fz{(const uint16_t*)x, K, K, (const uint16_t*)gamma, eps};
    const uint16_t* res = (const uint16_t*)residual;
    uint16_t* yy = (uint16_t*)y;
    const int T = act_tile_of(M);
    switch (epilogue) {
      case BITNET_EPI_NONE: return dispatch_simt<EPI_NONE>(nullptr, nullptr, nullptr, M, Kp, T, w_packed, N, seg, res, yy, acc_out, stream, fz);
      case BITNET_EPI_RELU2_MUL: return dispatch_simt<EPI_RELU2_MUL>(nullptr, nullptr, nullptr, M, Kp, T, w_packed, N, seg, res, yy, acc_out, stream, fz);
      default: return dispatch_simt<EPI_RESIDUAL_ADD>(nullptr, nullptr, nullptr, M, Kp, T, w_packed, N, seg, res, yy, acc_out, stream, fz);
    }
  }
  if (int e = bitnet_act_quant(x, M, K, K, gamma, eps, q_ws, scale_ws, sum_ws, nullptr, stream)) return e;
  return bitnet_bitlinear_q(q_ws, scale_ws, sum_ws, M, K, w_packed, N, segments, epilogue, residual, y, acc_out,
                            path, stream);
}

size_t bitnet_gqa_decode_workspace_bytes(int B, int n_heads, int n_kv_heads, int max_ctx) {
  if (B <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || max_ctx <= 0) return 0;
  const int S = att_grid_splits(B, n_kv_heads, max_ctx);
  if (S <= 1) return 0;
  const size_t counters = ((size_t)B * n_kv_heads * sizeof(int) + 255) / 256 * 256;
  return counters + (size_t)B * n_kv_heads * S * att_part_floats(n_heads / n_kv_heads) * sizeof(float);
}

int bitnet_gqa_decode_attention(const void* qkv, int B, int n_heads, int n_kv_heads, int head_dim,
                                const int32_t* positions, const void* rope_cos, const void* rope_sin, int rope_len,
                                void* k_cache, void* v_cache, int max_len, int max_ctx, float scale, void* workspace,
                                size_t workspace_bytes, void* out, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!qkv || !positions || !rope_cos || !rope_sin || !k_cache || !v_cache || !out) return BITNET_ERR_INVALID_ARGUMENT;
  if (B <= 0 || n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads != 0 || head_dim != ATT_D || max_len <= 0 ||
      rope_len <= 0 || max_ctx < 0)
    return BITNET_ERR_INVALID_ARGUMENT;
  if (max_ctx == 0) max_ctx = std::min(max_len, rope_len);
  if (max_ctx > max_len || max_ctx > rope_len) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(qkv, 4) || !aligned(out, 2))
    return BITNET_ERR_ALIGNMENT;
  const size_t ws_need = bitnet_gqa_decode_workspace_bytes(B, n_heads, n_kv_heads, max_ctx);
  if (ws_need > 0 && (workspace == nullptr || workspace_bytes < ws_need)) return BITNET_ERR_INVALID_ARGUMENT;
  if (ws_need > 0 && !aligned(workspace, 16)) return BITNET_ERR_ALIGNMENT;
  AttnParams p;
  p.qkv = (const uint16_t*)qkv;
  p.n_heads = n_heads;
  p.n_kv = n_kv_heads;
  p.G = n_heads / n_kv_heads;
  p.positions = positions;
  p.rope_cos = (const uint16_t*)rope_cos;
  p.rope_sin = (const uint16_t*)rope_sin;
  p.rope_len = rope_len;
  p.k_cache = (uint16_t*)k_cache;
  p.v_cache = (uint16_t*)v_cache;
  p.max_len = max_len;
  p.max_ctx = max_ctx;
  p.nsplit = att_grid_splits(B, n_kv_heads, max_ctx);
  p.prefetch = att_prefetch_pays(B, n_kv_heads, max_ctx);
  p.scale = scale;
  const size_t counters = ((size_t)B * n_kv_heads * sizeof(int) + 255) / 256 * 256;
  p.ws_count = ws_need > 0 ? (int*)workspace : nullptr;
  p.ws_part = ws_need > 0 ? (float*)((uint8_t*)workspace + counters) : nullptr;
  p.out = (uint16_t*)out;
  const dim3 grid(B, n_kv_heads, p.nsplit), block(ATT_THREADS);
  const size_t smem = att_smem_bytes(p.G);
  switch (p.G) {
    case 1:
      if (int e = ensure_smem(gqa_decode_kernel<1>, &g_smem_att[0])) return e;
      return launch(gqa_decode_kernel<1>, grid, block, smem, stream, 1, p);
    case 2:
      if (int e = ensure_smem(gqa_decode_kernel<2>, &g_smem_att[1])) return e;
      return launch(gqa_decode_kernel<2>, grid, block, smem, stream, 1, p);
    case 4:
      if (int e = ensure_smem(gqa_decode_kernel<4>, &g_smem_att[2])) return e;
      return launch(gqa_decode_kernel<4>, grid, block, smem, stream, 1, p);
    case 8:
      if (int e = ensure_smem(gqa_decode_kernel<8>, &g_smem_att[3])) return e;
      return launch(gqa_decode_kernel<8>, grid, block, smem, stream, 1, p);
    default: return BITNET_ERR_INVALID_ARGUMENT;
  }
}

static int rope_prefill_impl(const void* qkv, int B, int P, const int32_t* cu, int tokens, int n_heads,
                             int n_kv_heads, int head_dim, const void* rope_cos, const void* rope_sin, int rope_len,
                             void* q_out, void* k_cache, void* v_cache, int max_len, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!qkv || !rope_cos || !rope_sin || !q_out || !k_cache || !v_cache) return BITNET_ERR_INVALID_ARGUMENT;
  if (B <= 0 || P <= 0 || tokens <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 ||
      head_dim != ATT_D || P > max_len || P > rope_len)
    return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(qkv, 4) || !aligned(q_out, 4) || !aligned(k_cache, 4) || !aligned(v_cache, 4) || !aligned(rope_cos, 4) ||
      !aligned(rope_sin, 4) || (cu && !aligned(cu, 4)))
    return BITNET_ERR_ALIGNMENT;
  RopePrefillParams p;
  memset(&p, 0, sizeof(p));
  p.qkv = (const uint16_t*)qkv;
  p.B = B;
  p.P = P;
  p.n_heads = n_heads;
  p.n_kv = n_kv_heads;
  p.cu = cu;
  p.rope_len = rope_len;
  p.rope_cos = (const uint16_t*)rope_cos;
  p.rope_sin = (const uint16_t*)rope_sin;
  p.q_out = (uint16_t*)q_out;
  p.k_cache = (uint16_t*)k_cache;
  p.v_cache = (uint16_t*)v_cache;
  p.max_len = max_len;
  // 16-byte accesses when every pointer allows them (the row strides are multiples of 256 bytes)
  if (aligned(qkv, 16) && aligned(q_out, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) &&
      aligned(rope_cos, 16) && aligned(rope_sin, 16))
    return launch(rope_append_prefill_vec_kernel, dim3((tokens + RPF_TOK - 1) / RPF_TOK), dim3(256), 0, stream, 1,
                  p, tokens);
  return launch(rope_append_prefill_kernel, dim3(tokens), dim3(256), 0, stream, 1, p);
}

int bitnet_rope_append_prefill(const void* qkv, int B, int P, int n_heads, int n_kv_heads, int head_dim,
                               const void* rope_cos, const void* rope_sin, int rope_len, void* q_out, void* k_cache,
                               void* v_cache, int max_len, bitnet_stream_t stream) {
  if (B <= 0 || P <= 0 || (long long)B * P > 0x7fffffffLL) return BITNET_ERR_INVALID_ARGUMENT;
  return rope_prefill_impl(qkv, B, P, nullptr, B * P, n_heads, n_kv_heads, head_dim, rope_cos, rope_sin, rope_len,
                           q_out, k_cache, v_cache, max_len, stream);
}

int bitnet_rope_append_prefill_varlen(const void* qkv, int B, const int32_t* cu_seqlens, int total_tokens,
                                      int max_seqlen, int n_heads, int n_kv_heads, int head_dim,
                                      const void* rope_cos, const void* rope_sin, int rope_len, void* q_out,
                                      void* k_cache, void* v_cache, int max_len, bitnet_stream_t stream) {
  if (!cu_seqlens) return BITNET_ERR_INVALID_ARGUMENT;
  return rope_prefill_impl(qkv, B, max_seqlen, cu_seqlens, total_tokens, n_heads, n_kv_heads, head_dim, rope_cos,
                           rope_sin, rope_len, q_out, k_cache, v_cache, max_len, stream);
}

static int attention_prefill_impl(const void* q, const void* k_cache, const void* v_cache, int B, int P,
                                  const int32_t* cu, int n_heads, int n_kv_heads, int head_dim, int max_len,
                                  float scale, void* out, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!q || !k_cache || !v_cache || !out) return BITNET_ERR_INVALID_ARGUMENT;
  if (B <= 0 || P <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || head_dim != ATT_D ||
      P > max_len || B > 65535)
    return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(q, 4) || !aligned(out, 4) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || (cu && !aligned(cu, 4)))
    return BITNET_ERR_ALIGNMENT;
  if (int e = ensure_smem(attention_prefill_kernel, &g_smem_apf)) return e;
  AttnPrefillParams p;
  memset(&p, 0, sizeof(p));
  p.q = (const uint16_t*)q;
  p.k_cache = (const uint16_t*)k_cache;
  p.v_cache = (const uint16_t*)v_cache;
  p.B = B;
  p.P = P;
  p.n_heads = n_heads;
  p.n_kv = n_kv_heads;
  p.max_len = max_len;
  p.scale = scale;
  p.out = (uint16_t*)out;
  p.cu = cu;
  return launch(attention_prefill_kernel, dim3((P + APF_QB - 1) / APF_QB, n_heads, B), dim3(APF_THREADS), APF_SMEM,
                stream, 1, p);
}

int bitnet_attention_prefill(const void* q, const void* k_cache, const void* v_cache, int B, int P, int n_heads,
                             int n_kv_heads, int head_dim, int max_len, float scale, void* out,
                             bitnet_stream_t stream) {
  return attention_prefill_impl(q, k_cache, v_cache, B, P, nullptr, n_heads, n_kv_heads, head_dim, max_len, scale, out,
                                stream);
}

int bitnet_attention_prefill_varlen(const void* q, const void* k_cache, const void* v_cache, int B,
                                    const int32_t* cu_seqlens, int max_seqlen, int n_heads, int n_kv_heads,
                                    int head_dim, int max_len, float scale, void* out, bitnet_stream_t stream) {
  if (!cu_seqlens) return BITNET_ERR_INVALID_ARGUMENT;
  return attention_prefill_impl(q, k_cache, v_cache, B, max_seqlen, cu_seqlens, n_heads, n_kv_heads, head_dim,
                                max_len, scale, out, stream);
}

size_t bitnet_lm_head_bytes(int V, int K) {
  if (V <= 0 || K <= 0) return 0;
  return (size_t)round_up(V, 128) * (size_t)round_up(K, 8) * 2;
}

int bitnet_pack_lm_head(const void* w, int V, int K, void* w_tiled, bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!w || !w_tiled || V <= 0 || K <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(w_tiled, 16) || !aligned(w, 2)) return BITNET_ERR_ALIGNMENT;
  const int Vpad = round_up(V, 128), KC8 = round_up(K, 8) / 8;
  pack_lm_head_kernel<<<grid_for((size_t)Vpad * KC8, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)w, V, K, Vpad, KC8, (uint4*)w_tiled);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BITNET_OK : cuda_fail(e, "kernel launch");
}

int bitnet_embed_gather(const int32_t* ids, int B, const void* w_tiled, int V, int K, void* out,
                        bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!ids || !w_tiled || !out || B <= 0 || V <= 0 || K <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(w_tiled, 16) || !aligned(out, 2)) return BITNET_ERR_ALIGNMENT;
  const int KC8 = round_up(K, 8) / 8;
  return launch(embed_gather_kernel, dim3((KC8 + 127) / 128, B), dim3(128), 0, stream, 1, ids, B,
                (const uint4*)w_tiled, V, K, KC8, (uint16_t*)out);
}

// Workspace of bitnet_lm_head_argmax: the per-CTA (max, index) pairs
// (<= kMaxLmGrid CTAs), then the hidden states in the tiled tcgen05 layout.
constexpr int kMaxLmGrid = 160;
static size_t lm_ws_hidden_offset(int B) { return (lm_head_part_bytes(B, kMaxLmGrid) + 255) / 256 * 256; }

size_t bitnet_argmax_workspace_bytes(int B, int K, int V) {
  if (B <= 0 || V <= 0 || K <= 0 || B > 256) return 0;
  return lm_ws_hidden_offset(B) + (size_t)(round_up(K, 8) / 8) * lm_head_tile_T(B) * 16;
}

// tile_hidden + lm_head_tc; the per-CTA pairs are left in the workspace.
static int lm_head_pairs(const void* h, int B, int K, const void* w_tiled, int V, void* workspace, void* logits_out,
                         bitnet_stream_t stream, int* grid_out) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!h || !w_tiled || !workspace || B <= 0 || B > 256 || V <= 0 || K <= 0 || (K % 16) != 0)
    return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(w_tiled, 16) || !aligned(workspace, 256) || !aligned(h, 2)) return BITNET_ERR_ALIGNMENT;
  const int K8 = round_up(K, 8) / 8, ntiles = round_up(V, 128) / 128, T = lm_head_tile_T(B);
  const int grid = ntiles < d->sms ? ntiles : (d->sms < kMaxLmGrid ? d->sms : kMaxLmGrid);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ArgPair* part = reinterpret_cast<ArgPair*>(ws);
  uint8_t* h_tiled = ws + lm_ws_hidden_offset(B);
  if (int e = launch(tile_hidden_kernel, dim3((K8 * T + 255) / 256), dim3(256), 0, stream, 1, (const uint16_t*)h, B,
                     K, T, K8, reinterpret_cast<uint4*>(h_tiled)))
    return e;
  if (int e = ensure_smem(lm_head_tc_kernel, &g_smem_lmh)) return e;
  const int slot = lmt_slot_bytes(T);
  const int nstage_total = ((K8 + LMT_STAGE_CHUNKS - 1) / LMT_STAGE_CHUNKS) * ((ntiles + grid - 1) / grid);
  int nslot = (int)((kMaxDynSmem - lmt_ctrl_bytes()) / slot);
  if (nslot > LMT_MAX_SLOTS) nslot = LMT_MAX_SLOTS;
  if (nslot > nstage_total) nslot = nstage_total;
  if (nslot < 2) return BITNET_ERR_INVALID_ARGUMENT;
  LmTcParams p;
  p.w = (const uint8_t*)w_tiled;
  p.h = h_tiled;
  p.B = B;
  p.T = T;
  p.K8 = K8;
  p.V = V;
  p.ntiles = ntiles;
  p.nslot = nslot;
  p.part = part;
  p.logits = (uint16_t*)logits_out;
  const size_t smem = (size_t)lmt_ctrl_bytes() + (size_t)nslot * slot;
  *grid_out = grid;
  return launch(lm_head_tc_kernel, dim3(grid), dim3(LMT_THREADS), smem, stream, 1, p);
}

int bitnet_lm_head_argmax(const void* h, int B, int K, const void* w_tiled, int V, void* workspace, int32_t* out_ids,
                          void* logits_out, int32_t* advance_positions, bitnet_stream_t stream) {
  if (!out_ids) return BITNET_ERR_INVALID_ARGUMENT;
  int grid = 0;
  if (int e = lm_head_pairs(h, B, K, w_tiled, V, workspace, logits_out, stream, &grid)) return e;
  return launch(argmax_reduce_kernel, dim3(B), dim3(256), 0, stream, 1, (const ArgPair*)workspace, grid, B, out_ids,
                advance_positions, (ArgPair*)nullptr, 0);
}

int bitnet_lm_head_argmax_shard(const void* h, int B, int K, const void* w_tiled_shard, int V_shard,
                                int vocab_offset, void* workspace, void* pairs_out, bitnet_stream_t stream) {
  if (!pairs_out || vocab_offset < 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(pairs_out, 8)) return BITNET_ERR_ALIGNMENT;
  int grid = 0;
  if (int e = lm_head_pairs(h, B, K, w_tiled_shard, V_shard, workspace, nullptr, stream, &grid)) return e;
  return launch(argmax_reduce_kernel, dim3(B), dim3(256), 0, stream, 1, (const ArgPair*)workspace, grid, B,
                (int32_t*)nullptr, (int32_t*)nullptr, (ArgPair*)pairs_out, vocab_offset);
}

int bitnet_argmax_merge_pairs(const void* pairs, int nshard, int B, int32_t* out_ids, int32_t* advance_positions,
                              bitnet_stream_t stream) {
  DevInfo* d;
  if (int e = device_info(&d)) return e;
  if (!pairs || !out_ids || nshard <= 0 || B <= 0 || B > 256) return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(pairs, 8)) return BITNET_ERR_ALIGNMENT;
  return launch(argmax_reduce_kernel, dim3(B), dim3(256), 0, stream, 1, (const ArgPair*)pairs, nshard, B, out_ids,
                advance_positions, (ArgPair*)nullptr, 0);
}

}  // extern "C"

// ===========================================================================
// BitLinear without any caller-provided scratch (bitnet_bitlinear_noalloc).
//
// For callers that cannot allocate device memory at the point of the call --
// e.g. an FFI host (cgo, JNI, a C plugin) that holds no CUDA allocator of its
// own, or code running where allocation is forbidden -- the int8 activations,
// row scales and row sums of bitnet_bitlinear live in one file-scope device
// array instead of in buffers the caller passes in.  The array is part of the
// library image: every GPU that loads the library holds it until the process
// exits.
//
// Limits: act_rows(M) <= BITNET_NOALLOC_MAX_ROWS and
// act_rows(M) * round_up(K, 64) <= BITNET_NOALLOC_MAX_ACT_BYTES.
// Nothing in the array has to start at zero: every call's quantisation kernel
// writes all of it that the same call's BitLinear kernel reads.
// All calls share the array, so two calls whose kernels overlap on the GPU
// (different streams, or different host threads) race on it.
// ===========================================================================
namespace {

constexpr size_t kNoallocQBytes = BITNET_NOALLOC_MAX_ACT_BYTES;
constexpr int kNoallocRows = BITNET_NOALLOC_MAX_ROWS;
constexpr size_t kNoallocScaleOff = kNoallocQBytes;
constexpr size_t kNoallocSumOff = kNoallocScaleOff + (size_t)kNoallocRows * sizeof(float);
constexpr size_t kNoallocBytes = kNoallocSumOff + (size_t)kNoallocRows * sizeof(int32_t);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per
// device with that device current and the looked-up pointer is what the
// kernels receive.
// Published with release / read with acquire, so a thread that sees a
// non-null pointer also sees the completed look-up (double-checked locking
// without a data race).
std::atomic<unsigned char*> g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return BITNET_ERR_INVALID_ARGUMENT;
  unsigned char* ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    ptr = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (ptr == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
      ptr = static_cast<unsigned char*>(p);
      g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return BITNET_OK;
}

}  // namespace

extern "C" int bitnet_bitlinear_noalloc(const void* x, int M, int K, const void* gamma, float eps,
                                        const uint8_t* w_packed, int N, const bitnet_segments_t* segments,
                                        int epilogue, const void* residual, void* y, int32_t* acc_out, int path,
                                        bitnet_stream_t stream) {
  if (M <= 0 || K <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  const int rows = act_rows_of(M);
  if (rows > kNoallocRows || (size_t)rows * (size_t)round_up(K, 64) > kNoallocQBytes)
    return BITNET_ERR_SCRATCH_LIMIT;
  unsigned char* base = nullptr;
  if (int e = noalloc_scratch(&base)) return e;
  int8_t* q = reinterpret_cast<int8_t*>(base);
  float* scale = reinterpret_cast<float*>(base + kNoallocScaleOff);
  int32_t* sum = reinterpret_cast<int32_t*>(base + kNoallocSumOff);
  return bitnet_bitlinear(x, M, K, gamma, eps, w_packed, N, segments, epilogue, residual, y, acc_out, q, scale, sum,
                          path, stream);
}

// ---------------------------------------------------------------------------
// persistent decode of every layer
// ---------------------------------------------------------------------------
static_assert(sizeof(void*) != 8 || sizeof(bitnet_decode_layer_t) == 224, "bitnet_decode_layer_t layout");
static_assert(sizeof(void*) != 8 || sizeof(bitnet_decode_desc_t) == 144, "bitnet_decode_desc_t layout");

struct bitnet_decode_plan {
  int device = -1;
  int G = 0;
  int grid = 0;
  size_t smem = 0;
  MkParams p;
  void* dev_block = nullptr;  // layers | codes | split-K scratch | barrier words (one allocation)
};

namespace {
std::atomic<unsigned long long> g_smem_mk[4];

int mk_split(int NT, int KC, int grid) {
  int best = 1;
  for (int s = 1; s <= 8 && s <= KC; ++s)
    if (NT * s <= grid) best = s;
  return best;
}

template <int G>
int mk_launch(bitnet_decode_plan* pl, cudaStream_t st) {
  if (int e = ensure_smem(decode_layers_kernel<G>, &g_smem_mk[G == 1 ? 0 : (G == 2 ? 1 : (G == 4 ? 2 : 3))]))
    return e;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(pl->grid);
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = pl->smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_layers_kernel<G>, pl->p);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(decode_layers)");
  return BITNET_OK;
}

template <int G>
int mk_occupancy(int* blocks, size_t smem) {
  if (int e = ensure_smem(decode_layers_kernel<G>, &g_smem_mk[G == 1 ? 0 : (G == 2 ? 1 : (G == 4 ? 2 : 3))]))
    return e;
  const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, decode_layers_kernel<G>, MK_THREADS, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  return BITNET_OK;
}
}  // namespace

extern "C" int bitnet_decode_plan_create(const bitnet_decode_desc_t* d, bitnet_decode_plan_t** out) {
  if (!d || !out) return BITNET_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  DevInfo* di;
  if (int e = device_info(&di)) return e;
  const int L = d->num_layers, B = d->batch, H = d->hidden, F = d->intermediate, NH = d->n_heads, NKV = d->n_kv_heads;
  if (L <= 0 || B <= 0 || B > MK_MAX_T || H <= 0 || F <= 0 || NH <= 0 || NKV <= 0 || NH % NKV != 0 ||
      d->head_dim != ATT_D || !d->layers)
    return BITNET_ERR_INVALID_ARGUMENT;
  const int G = NH / NKV;
  if (G != 1 && G != 2 && G != 4 && G != 8) return BITNET_ERR_INVALID_ARGUMENT;
  const int AK = NH * ATT_D;  // attention output width
  for (int k : {H, F, AK})
    if (k % 8 != 0 || round_up(k, 64) > 8 * AQ_THREADS * AQ_MAXC) return BITNET_ERR_INVALID_ARGUMENT;
  if (!d->hidden_state || !d->qkv || !d->attn || !d->mid || !d->positions || !d->rope_cos || !d->rope_sin)
    return BITNET_ERR_INVALID_ARGUMENT;
  if (!aligned(d->hidden_state, 16) || !aligned(d->qkv, 16) || !aligned(d->attn, 16) || !aligned(d->mid, 16))
    return BITNET_ERR_ALIGNMENT;
  int max_ctx = d->max_ctx;
  if (max_ctx < 0 || d->max_len <= 0 || d->rope_len <= 0) return BITNET_ERR_INVALID_ARGUMENT;
  if (max_ctx == 0) max_ctx = std::min(d->max_len, d->rope_len);
  if (max_ctx > d->max_len || max_ctx > d->rope_len) return BITNET_ERR_INVALID_ARGUMENT;
  const size_t att_ws = bitnet_gqa_decode_workspace_bytes(B, NH, NKV, max_ctx);
  if (att_ws > 0 && (!d->attn_workspace || d->attn_workspace_bytes < att_ws)) return BITNET_ERR_INVALID_ARGUMENT;
  if (att_ws > 0 && !aligned(d->attn_workspace, 16)) return BITNET_ERR_ALIGNMENT;

  auto* pl = new bitnet_decode_plan();
  cudaGetDevice(&pl->device);
  pl->G = G;
  MkParams& p = pl->p;
  memset(&p, 0, sizeof(p));
  p.L = L;
  p.B = B;
  p.T = act_tile_of(B);
  p.eps = d->eps;
  const int shapes[4][3] = {{(NH + 2 * NKV) * ATT_D, H, BITNET_EPI_NONE},
                            {H, AK, BITNET_EPI_RESIDUAL_ADD},
                            {2 * F, H, BITNET_EPI_RELU2_MUL},
                            {H, F, BITNET_EPI_RESIDUAL_ADD}};
  pl->smem = mk_smem_bytes(G);
  int occ = 0;
  int e = 0;
  switch (G) {
    case 1: e = mk_occupancy<1>(&occ, pl->smem); break;
    case 2: e = mk_occupancy<2>(&occ, pl->smem); break;
    case 4: e = mk_occupancy<4>(&occ, pl->smem); break;
    default: e = mk_occupancy<8>(&occ, pl->smem); break;
  }
  if (e || occ < 1) {
    delete pl;
    return e ? e : BITNET_ERR_UNSUPPORTED_DEVICE;
  }
  pl->grid = di->sms;  // one CTA per SM, all resident
  int max_nt = 1;
  for (int i = 0; i < 4; ++i) {
    MkBl& bl = p.bl[i];
    bl.N = shapes[i][0];
    bl.K = shapes[i][1];
    bl.epi = shapes[i][2];
    bl.KC = round_up(bl.K, 64) / 64;
    bl.NT = round_up(bl.N, 128) / 128;
    bl.S = d->splits[i] > 0 ? std::min(d->splits[i], bl.KC) : mk_split(bl.NT, bl.KC, pl->grid);
    if (bl.S > 1) max_nt = std::max(max_nt, bl.NT);
  }
  // device block: layers | q_h | q_f | s_h rs_h s_f rs_f | acc_ws | tile_cnt | barrier words
  const int T = p.T;
  const size_t kph = (size_t)round_up(std::max(H, AK), 64), kpf = (size_t)round_up(F, 64);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_layers = take(sizeof(MkLayer) * L);
  const size_t o_qh = take((size_t)T * kph), o_qf = take((size_t)T * kpf);
  const size_t o_sh = take(4 * T), o_rsh = take(4 * T), o_sf = take(4 * T), o_rsf = take(4 * T);
  const size_t o_acc = take((size_t)max_nt * T * 128 * 4), o_cnt = take((size_t)max_nt * 4);
  const size_t o_sync = take(256);
  cudaError_t ce = cudaMalloc(&pl->dev_block, off);
  if (ce != cudaSuccess) {
    delete pl;
    return cuda_fail(ce, "cudaMalloc(decode plan)");
  }
  uint8_t* base = (uint8_t*)pl->dev_block;
  ce = cudaMemset(base, 0, off);
  std::vector<MkLayer> layers(L);
  for (int l = 0; l < L && ce == cudaSuccess; ++l) {
    const bitnet_decode_layer_t& s = d->layers[l];
    MkLayer& m = layers[l];
    m.w[0] = s.w_qkv;
    m.w[1] = s.w_o;
    m.w[2] = s.w_gate_up;
    m.w[3] = s.w_down;
    const bitnet_segments_t* segs[4] = {&s.seg_qkv, &s.seg_o, &s.seg_gate_up, &s.seg_down};
    for (int i = 0; i < 4; ++i) {
      if (!m.w[i] || !aligned(m.w[i], 16)) e = BITNET_ERR_ALIGNMENT;
      if (!e) e = to_dev_segments(segs[i], p.bl[i].N, p.bl[i].epi, &m.seg[i]);
    }
    m.gamma[0] = (const uint16_t*)s.input_layernorm;
    m.gamma[1] = (const uint16_t*)s.attn_sub_norm;
    m.gamma[2] = (const uint16_t*)s.post_attention_layernorm;
    m.gamma[3] = (const uint16_t*)s.ffn_sub_norm;
    for (int i = 0; i < 4; ++i)
      if (m.gamma[i] && !aligned(m.gamma[i], 16)) e = BITNET_ERR_ALIGNMENT;
    m.k_cache = (uint16_t*)s.k_cache;
    m.v_cache = (uint16_t*)s.v_cache;
    if (!m.k_cache || !m.v_cache) e = BITNET_ERR_INVALID_ARGUMENT;
    else if (!aligned(m.k_cache, 16) || !aligned(m.v_cache, 16)) e = BITNET_ERR_ALIGNMENT;
  }
  if (ce == cudaSuccess && !e) ce = cudaMemcpy(base + o_layers, layers.data(), sizeof(MkLayer) * L, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess || e) {
    cudaFree(pl->dev_block);
    delete pl;
    return e ? e : cuda_fail(ce, "decode plan set-up");
  }
  p.layers = (const MkLayer*)(base + o_layers);
  p.hidden = (uint16_t*)d->hidden_state;
  p.qkv = (uint16_t*)d->qkv;
  p.attn = (uint16_t*)d->attn;
  p.mid = (uint16_t*)d->mid;
  p.q_h = (int8_t*)(base + o_qh);
  p.q_f = (int8_t*)(base + o_qf);
  p.s_h = (float*)(base + o_sh);
  p.rs_h = (int32_t*)(base + o_rsh);
  p.s_f = (float*)(base + o_sf);
  p.rs_f = (int32_t*)(base + o_rsf);
  p.acc_ws = (int32_t*)(base + o_acc);
  p.tile_cnt = (int*)(base + o_cnt);
  p.sync_ctr = (unsigned*)(base + o_sync);
  p.abort_flag = (int*)(base + o_sync + 4);
  AttnParams& a = p.att;
  a.qkv = p.qkv;
  a.n_heads = NH;
  a.n_kv = NKV;
  a.G = G;
  a.positions = d->positions;
  a.rope_cos = (const uint16_t*)d->rope_cos;
  a.rope_sin = (const uint16_t*)d->rope_sin;
  a.rope_len = d->rope_len;
  a.max_len = d->max_len;
  a.max_ctx = max_ctx;
  a.nsplit = att_grid_splits(B, NKV, max_ctx);
  a.prefetch = 0;  // the persistent kernel has no launch to overlap
  a.scale = 1.0f / sqrtf((float)ATT_D);
  const size_t counters = ((size_t)B * NKV * sizeof(int) + 255) / 256 * 256;
  a.ws_count = att_ws > 0 ? (int*)d->attn_workspace : nullptr;
  a.ws_part = att_ws > 0 ? (float*)((uint8_t*)d->attn_workspace + counters) : nullptr;
  a.out = p.attn;
  p.att_units = B * NKV * a.nsplit;
  *out = pl;
  return BITNET_OK;
}

extern "C" int bitnet_decode_plan_run(bitnet_decode_plan_t* pl, bitnet_stream_t stream) {
  if (!pl) return BITNET_ERR_INVALID_ARGUMENT;
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != pl->device) return BITNET_ERR_INVALID_ARGUMENT;
  const cudaError_t ce = cudaMemsetAsync(pl->p.sync_ctr, 0, 8, (cudaStream_t)stream);  // barrier + abort words
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaMemsetAsync(decode barrier)");
  switch (pl->G) {
    case 1: return mk_launch<1>(pl, (cudaStream_t)stream);
    case 2: return mk_launch<2>(pl, (cudaStream_t)stream);
    case 4: return mk_launch<4>(pl, (cudaStream_t)stream);
    default: return mk_launch<8>(pl, (cudaStream_t)stream);
  }
}

extern "C" int bitnet_decode_plan_destroy(bitnet_decode_plan_t* pl) {
  if (!pl) return BITNET_OK;
  cudaFree(pl->dev_block);
  delete pl;
  return BITNET_OK;
}
