// Fused RMSNorm + per-token int8 absmax activation quantisation.
//
// Semantics (one token row x of K bf16 values, gamma bf16 or absent):
//   ss     = sum_k x_k^2                         accumulated in fp64
//   var    = fp32(ss / K)
//   r      = 1 / sqrt(var + eps)                 fp32, IEEE sqrt and divide
//   y_k    = bf16(x_k * r)                       HF BitNetRMSNorm: fp32 math, cast to bf16,
//   a_k    = bf16(gamma_k * y_k)                 then weight * hidden in bf16
//   amax   = max(max_k |a_k|, 1e-5)
//   s      = 127 / amax                          (row_scale)
//   q_k    = clamp(rint(a_k * s), -128, 127)     half-to-even, as np.round / torch.round
//   sum    = sum_k q_k                           (row_sum, used by the ternary epilogue)
// Without gamma, a_k = x_k.  Every fp32 operation is an explicit _rn intrinsic so
// the compiler cannot contract or reorder it.  A square of a bf16 value has at
// most 16 significant bits, so the fp64 sum of K of them is exact in any order
// when the largest square is at most 2^(37 - ceil(log2 K)) times the smallest
// nonzero one (|x| spanning 2^12 at K = 2560): the codes then cannot depend on
// the reduction tree.  Beyond that span the sum may round, and two orders can
// differ in the last bits of ss; var = fp32(ss / K) still agrees unless ss / K
// lies within ~2^-29 (relative) of an fp32 rounding boundary.
#pragma once
#include "common.cuh"

namespace bitnet {

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* scratch, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // protect scratch from a previous use
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  T r = scratch[0];
  for (int i = 1; i < nw; ++i) r = op(r, scratch[i]);
  return r;
}

struct OpAddD { __device__ double operator()(double a, double b) const { return a + b; } };
struct OpMaxF { __device__ float operator()(float a, float b) const { return fmaxf(a, b); } };
struct OpAddI { __device__ int operator()(int a, int b) const { return a + b; } };

// grid = act_rows(M) (one CTA per padded token row), block = 256,
// dynamic smem = Kp * 4 bytes.
__global__ void __launch_bounds__(256)
act_quant_kernel(const uint16_t* __restrict__ x, int M, int K, int ldx, const uint16_t* __restrict__ gamma,
                 float eps, int8_t* __restrict__ q, float* __restrict__ row_scale, int32_t* __restrict__ row_sum,
                 uint16_t* __restrict__ normed_out, int T, int Kp) {
  extern __shared__ float sval[];
  __shared__ double red_d[32];
  __shared__ float red_f[32];
  __shared__ int red_i[32];

  // Let the next kernel launch now (it waits for this grid to complete before
  // it reads anything this grid writes); this grid waits for its predecessor.
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  const bool valid = m < M;

  double ss = 0.0;
  for (int k = tid; k < Kp; k += nt) {
    float v = 0.f;
    if (valid && k < K) v = bf16_bits_to_f32(x[(size_t)m * ldx + k]);
    sval[k] = v;
    ss += (double)v * (double)v;
  }

  if (gamma != nullptr) {
    ss = block_reduce(ss, red_d, OpAddD());
    const float var = __double2float_rn(__ddiv_rn(ss, (double)K));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int k = tid; k < K; k += nt) {
      const float y = round_bf16(__fmul_rn(sval[k], r));
      sval[k] = round_bf16(__fmul_rn(bf16_bits_to_f32(gamma[k]), y));
    }
  }
  __syncthreads();

  if (normed_out != nullptr && valid) {
    for (int k = tid; k < K; k += nt) normed_out[(size_t)m * K + k] = f32_to_bf16_bits(sval[k]);
  }
  if (q == nullptr) return;

  float amax = 0.f;
  for (int k = tid; k < K; k += nt) amax = fmaxf(amax, fabsf(sval[k]));
  amax = block_reduce(amax, red_f, OpMaxF());
  amax = fmaxf(amax, 1e-5f);
  const float s = __fdiv_rn(127.0f, amax);

  int qsum = 0;
  for (int k4 = tid * 4; k4 < Kp; k4 += nt * 4) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = k4 + i;
      int qi = 0;
      if (valid && k < K) {
        qi = __float2int_rn(__fmul_rn(sval[k], s));
        qi = max(-128, min(127, qi));
      }
      qsum += qi;
      word |= ((uint32_t)(qi & 0xFF)) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(q + alayout_offset(m, k4, T, Kp)) = word;
  }
  qsum = block_reduce(qsum, red_i, OpAddI());
  if (tid == 0) {
    row_scale[m] = valid ? s : 1.0f;
    row_sum[m] = qsum;
  }
}

// Fast path: K % 8 == 0, 16-byte aligned rows (ldx % 8 == 0) and gamma, and
// K <= 8 * 256 * AQ_MAXC.  A row runs on 256 threads; each keeps up to
// AQ_MAXC 8-element chunks in registers (16-byte loads), and the three
// reductions use one barrier each (separate scratch words per reduction, so a
// reduction's scratch is never rewritten before every thread has read it).
// Same results as act_quant_kernel (the fp64 sum of squares is exact in any
// order; max and the integer sum are order-free).
constexpr int AQ_THREADS = 256;
constexpr int AQ_MAXC = 4;

__device__ __forceinline__ void aq_unpack8(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
  }
}

// Barrier over the row's 256 threads: __syncthreads (BAR == 0) or named barrier BAR.
template <int BAR>
__device__ __forceinline__ void aq_sync() {
  if (BAR == 0)
    __syncthreads();
  else
    named_bar_sync(BAR, AQ_THREADS);
}

struct AqScratch {
  double* d;  // [8]
  float* f;   // [8]
  int* i;     // [8]
};

template <int BAR, typename T, typename Op>
__device__ __forceinline__ T aq_allreduce(T v, T* scratch, Op op, int t) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((t & 31) == 0) scratch[t >> 5] = v;
  aq_sync<BAR>();
  T r = scratch[0];
#pragma unroll
  for (int i = 1; i < AQ_THREADS / 32; ++i) r = op(r, scratch[i]);
  return r;
}

// gamma chunks of thread t, kept packed (bf16 x 8 per register quad); gamma
// does not come from the previous kernel, so the standalone kernel loads it
// before griddepcontrol.wait
__device__ __forceinline__ void aq_load_gamma(uint4 (&gr)[AQ_MAXC], const uint16_t* gamma, int K, int t) {
#pragma unroll
  for (int c = 0; c < AQ_MAXC; ++c) {
    const int ch = t + c * AQ_THREADS;
    gr[c] = (gamma != nullptr && ch < (K >> 3)) ? reinterpret_cast<const uint4*>(gamma)[ch] : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ uint4 aq_pack8(const float* f) {
  uint4 o;
  o.x = (uint32_t)f32_to_bf16_bits(f[0]) | ((uint32_t)f32_to_bf16_bits(f[1]) << 16);
  o.y = (uint32_t)f32_to_bf16_bits(f[2]) | ((uint32_t)f32_to_bf16_bits(f[3]) << 16);
  o.z = (uint32_t)f32_to_bf16_bits(f[4]) | ((uint32_t)f32_to_bf16_bits(f[5]) << 16);
  o.w = (uint32_t)f32_to_bf16_bits(f[6]) | ((uint32_t)f32_to_bf16_bits(f[7]) << 16);
  return o;
}

// RMSNorm of 8 values as HF computes it, bf16(gamma * bf16(x * r)), returned
// packed as bf16 (the form every later step reads).  Each rounding handles two
// values per conversion instruction.  In the one-row-per-CTA kernels (decode)
// it shortens the chain of dependent conversions (the decode step went from
// 1507 to 1471 us); in the many-row kernels it halves the load on the
// conversion pipe (those need launch bounds of two CTAs per SM: without them
// the helpers raise the register count past 128 and one CTA fits per SM).
__device__ __forceinline__ uint32_t aq_norm2(uint32_t x, uint32_t g, uint64_t rr) {
  const uint32_t y = f2_to_bf2(f2_mul(f2_from_bf2(x), rr));
  return f2_to_bf2(f2_mul(f2_from_bf2(g), f2_from_bf2(y)));
}
__device__ __forceinline__ uint4 aq_norm8(const uint4 xv, const uint4 gv, float r) {
  const uint64_t rr = f2_splat(r);
  return make_uint4(aq_norm2(xv.x, gv.x, rr), aq_norm2(xv.y, gv.y, rr), aq_norm2(xv.z, gv.z, rr),
                    aq_norm2(xv.w, gv.w, rr));
}

// rint(v), half to even, for |v| < 2^22 (the codes: |v| <= 127 plus rounding):
// adding 1.5 * 2^23 leaves rint(v) in the low mantissa bits of the sum.  The
// same result as __float2int_rn without the conversion pipe.
__device__ __forceinline__ int aq_rint_small(float v) {
  return __float_as_int(__fadd_rn(v, 12582912.0f)) - 0x4B400000;
}

// Row m (padded rows m >= M produce zero codes, scale 1, sum 0) on threads
// t = 0..255.  The row stays in registers as packed bf16: the input is bf16 and
// every normalised value is rounded to bf16, so repacking loses nothing.
template <int BAR>
__device__ void aq_row_vec(const uint16_t* __restrict__ x, int M, int K, int ldx, bool has_gamma,
                           const uint4 (&gr)[AQ_MAXC], float eps, int8_t* __restrict__ q,
                           float* __restrict__ row_scale, int32_t* __restrict__ row_sum,
                           uint16_t* __restrict__ normed_out, int T, int Kp, int m, const AqScratch& sc, int t) {
  const bool valid = m < M;
  const int KC8 = K >> 3;  // chunks of 8
  uint4 xr[AQ_MAXC];
#pragma unroll
  for (int c = 0; c < AQ_MAXC; ++c) {
    const int ch = t + c * AQ_THREADS;
    xr[c] = (valid && ch < KC8) ? reinterpret_cast<const uint4*>(x + (size_t)m * ldx)[ch] : make_uint4(0, 0, 0, 0);
  }
  if (has_gamma) {
    double ssp[4] = {0.0, 0.0, 0.0, 0.0};  // four independent chains (exact in any order)
#pragma unroll
    for (int c = 0; c < AQ_MAXC; ++c) {
      float f[8];
      aq_unpack8(xr[c], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ssp[e & 3] = fma((double)f[e], (double)f[e], ssp[e & 3]);
    }
    double ss = (ssp[0] + ssp[1]) + (ssp[2] + ssp[3]);
    ss = aq_allreduce<BAR>(ss, sc.d, OpAddD(), t);
    const float var = __double2float_rn(__ddiv_rn(ss, (double)K));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int c = 0; c < AQ_MAXC; ++c) {
      xr[c] = aq_norm8(xr[c], gr[c], r);
    }
  }
  if (normed_out != nullptr && valid) {
#pragma unroll
    for (int c = 0; c < AQ_MAXC; ++c) {
      const int ch = t + c * AQ_THREADS;
      if (ch < KC8) reinterpret_cast<uint4*>(normed_out + (size_t)m * K)[ch] = xr[c];
    }
  }
  if (q == nullptr) return;
  float amax = 0.f;
#pragma unroll
  for (int c = 0; c < AQ_MAXC; ++c) {
    float f[8];
    aq_unpack8(xr[c], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
  }
  amax = fmaxf(aq_allreduce<BAR>(amax, sc.f, OpMaxF(), t), 1e-5f);
  const float s = __fdiv_rn(127.0f, amax);
  int qsum = 0;
#pragma unroll
  for (int c = 0; c < AQ_MAXC; ++c) {
    const int ch = t + c * AQ_THREADS;
    if (ch * 8 < Kp) {  // chunks past K (up to Kp) are written as zeros
      float f[8];
      aq_unpack8(xr[c], f);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int qi = 0;
        if (valid && ch < KC8) qi = max(-128, min(127, aq_rint_small(__fmul_rn(f[e], s))));
        qsum += qi;
        if (e < 4)
          lo |= ((uint32_t)(qi & 0xFF)) << (8 * e);
        else
          hi |= ((uint32_t)(qi & 0xFF)) << (8 * (e - 4));
      }
      *reinterpret_cast<uint2*>(q + alayout_offset(m, ch * 8, T, Kp)) = make_uint2(lo, hi);
    }
  }
  qsum = aq_allreduce<BAR>(qsum, sc.i, OpAddI(), t);
  if (t == 0) {
    row_scale[m] = valid ? s : 1.0f;
    row_sum[m] = qsum;
  }
}

__global__ void __launch_bounds__(AQ_THREADS)
act_quant_vec_kernel(const uint16_t* __restrict__ x, int M, int K, int ldx, const uint16_t* __restrict__ gamma,
                     float eps, int8_t* __restrict__ q, float* __restrict__ row_scale, int32_t* __restrict__ row_sum,
                     uint16_t* __restrict__ normed_out, int T, int Kp) {
  __shared__ double red_d[AQ_THREADS / 32];
  __shared__ float red_f[AQ_THREADS / 32];
  __shared__ int red_i[AQ_THREADS / 32];
  pdl_trigger();
  uint4 gr[AQ_MAXC];
  aq_load_gamma(gr, gamma, K, threadIdx.x);
  pdl_wait();
  const AqScratch sc{red_d, red_f, red_i};
  aq_row_vec<0>(x, M, K, ldx, gamma != nullptr, gr, eps, q, row_scale, row_sum, normed_out, T, Kp, blockIdx.x, sc,
                threadIdx.x);
}

// Decode path (few rows): one CTA per token row with one thread per C chunks of
// 8 elements (blockDim = 32 * ceil(Kp / 8 / C / 32): 320 threads at K = 2560,
// 864 at K = 6912 with C = 1), so no thread carries empty chunks through the
// fp64 squares, the normalisation and the quantisation.  Every thread keeps
// its chunks in registers; the three reductions (fp64 sum of squares, max,
// integer sum) take one barrier each, with separate scratch so none is
// overwritten before every thread has read it.  Same arithmetic as aq_row_vec
// (bit-identical codes, scales, sums and normalised values).  Needs K % 8 == 0,
// 16-byte aligned rows (ldx % 8 == 0) and gamma, and Kp / 8 <= 1024 * C.
template <int C>
__global__ void __launch_bounds__(1024)
act_quant_row_kernel(const uint16_t* __restrict__ x, int M, int K, int ldx, const uint16_t* __restrict__ gamma,
                     float eps, int8_t* __restrict__ q, float* __restrict__ row_scale, int32_t* __restrict__ row_sum,
                     uint16_t* __restrict__ normed_out, int T, int Kp) {
  __shared__ double red_d[32];
  __shared__ float red_f[32];
  __shared__ int red_i[32];
  pdl_trigger();
  const int t = threadIdx.x, nt = blockDim.x, nw = nt >> 5, lane = t & 31, warp = t >> 5;
  const int KC8 = K >> 3;
  uint4 gr[C];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int ch = t + c * nt;
    gr[c] = (gamma != nullptr && ch < KC8) ? reinterpret_cast<const uint4*>(gamma)[ch] : make_uint4(0, 0, 0, 0);
  }
  pdl_wait();
  const int m = blockIdx.x;
  const bool valid = m < M;
  uint4 xr[C];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int ch = t + c * nt;
    xr[c] = (valid && ch < KC8) ? reinterpret_cast<const uint4*>(x + (size_t)m * ldx)[ch] : make_uint4(0, 0, 0, 0);
  }
  if (gamma != nullptr) {
    double ss0 = 0.0, ss1 = 0.0;  // two independent chains (exact in any order within the span condition)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      float f[8];
      aq_unpack8(xr[c], f);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        ss0 = fma((double)f[e], (double)f[e], ss0);
        ss1 = fma((double)f[e + 1], (double)f[e + 1], ss1);
      }
    }
    double ss = ss0 + ss1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red_d[warp] = ss;
    __syncthreads();
    ss = red_d[0];
    for (int i = 1; i < nw; ++i) ss += red_d[i];
    const float var = __double2float_rn(__ddiv_rn(ss, (double)K));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int c = 0; c < C; ++c) {
      xr[c] = aq_norm8(xr[c], gr[c], r);
    }
  }
  if (normed_out != nullptr && valid) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int ch = t + c * nt;
      if (ch < KC8) reinterpret_cast<uint4*>(normed_out + (size_t)m * K)[ch] = xr[c];
    }
  }
  if (q == nullptr) return;
  float amax = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float f[8];
    aq_unpack8(xr[c], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) red_f[warp] = amax;
  __syncthreads();
  amax = red_f[0];
  for (int i = 1; i < nw; ++i) amax = fmaxf(amax, red_f[i]);
  amax = fmaxf(amax, 1e-5f);
  const float s = __fdiv_rn(127.0f, amax);
  int qsum = 0;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int ch = t + c * nt;
    if (ch * 8 < Kp) {  // chunks past K (up to Kp) are written as zeros
      float f[8];
      aq_unpack8(xr[c], f);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int qi = 0;
        if (valid && ch < KC8) qi = max(-128, min(127, aq_rint_small(__fmul_rn(f[e], s))));
        qsum += qi;
        if (e < 4)
          lo |= ((uint32_t)(qi & 0xFF)) << (8 * e);
        else
          hi |= ((uint32_t)(qi & 0xFF)) << (8 * (e - 4));
      }
      *reinterpret_cast<uint2*>(q + alayout_offset(m, ch * 8, T, Kp)) = make_uint2(lo, hi);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
  if (lane == 0) red_i[warp] = qsum;
  __syncthreads();
  if (t == 0) {
    for (int i = 1; i < nw; ++i) qsum += red_i[i];
    row_scale[m] = valid ? s : 1.0f;
    row_sum[m] = qsum;
  }
}

// ---------------------------------------------------------------------------
// Many-row (prefill) arithmetic on packed bf16 pairs.  These kernels stream
// 16384 rows per launch and were bound by instruction issue and by the
// conversion pipe (one f32 -> bf16 conversion per rounding per value, a
// float -> int conversion per code, clamps and shift-or byte packing).  Per
// pair of values the helpers below use: shifts to widen bf16 to fp32, one
// paired conversion per rounding step, a bf16x2 max for the absmax, an add of
// 1.5 * 2^23 for the half-to-even rounding of the codes, byte permutes for the
// packing and dp4a for the row sum; the normalisation's fp32 products run as
// .f32x2 pairs (aq_norm8).  Results are bit-identical to aq_row_vec.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// x^2 of the two values of a packed pair, each added to its own fp64 chain
// (squares of bf16 values are exact in fp64).
__device__ __forceinline__ void aq_sq2(uint32_t v, double& a, double& b) {
  const double lo = (double)bf_lo(v), hi = (double)bf_hi(v);
  a = fma(lo, lo, a);
  b = fma(hi, hi, b);
}
__device__ __forceinline__ void aq_sq8(const uint4 v, double (&ss)[4]) {
  aq_sq2(v.x, ss[0], ss[1]);
  aq_sq2(v.y, ss[2], ss[3]);
  aq_sq2(v.z, ss[0], ss[1]);
  aq_sq2(v.w, ss[2], ss[3]);
}

// Packed |a| max: the magnitudes of bf16 values are non-negative, and max of
// two bf16x2 operands is exact.
__device__ __forceinline__ uint32_t aq_max2(uint32_t a, uint32_t b) {
  const __nv_bfloat162 r =
      __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t aq_absmax8(uint32_t m, const uint4 v) {
  const uint32_t mag = 0x7FFF7FFFu;
  const uint32_t t0 = aq_max2(v.x & mag, v.y & mag), t1 = aq_max2(v.z & mag, v.w & mag);
  return aq_max2(m, aq_max2(t0, t1));
}
// Row absmax of a warp from each lane's packed max (bits of non-negative bf16
// values order as the values do).
__device__ __forceinline__ float aq_warp_absmax(uint32_t m) {
  const uint32_t b = max(m & 0xFFFFu, m >> 16);
  return __uint_as_float(__reduce_max_sync(0xffffffffu, b) << 16);
}

// Codes of four normalised values (two packed pairs): q = rint(a * s) half to
// even, as the low byte of fp32(a * s) + 1.5 * 2^23 (that sum holds
// 0x4B400000 + q, whose low byte is q mod 256).  No clamp: |a| <= amax and
// s = fp32(127 / amax) give |fp32(a * s)| <= 127 (1 + 2^-24)^2 < 127.5, so
// q lies in [-127, 127] for finite inputs.
// The product and the add stay scalar: issued as a .f32x2 multiply followed
// by a .f32x2 add they gave rint of the exact product (33 of 38,400 codes one
// off at near-ties, measured on B200), not rint(fp32(a * s)).
__device__ __forceinline__ uint32_t aq_code_bits(float a, float s) {
  return __float_as_uint(__fadd_rn(__fmul_rn(a, s), 12582912.0f));
}
__device__ __forceinline__ uint32_t aq_codes4(uint32_t a01, uint32_t a23, float s) {
  const uint32_t lo = __byte_perm(aq_code_bits(bf_lo(a01), s), aq_code_bits(bf_hi(a01), s), 0x0040);
  const uint32_t hi = __byte_perm(aq_code_bits(bf_lo(a23), s), aq_code_bits(bf_hi(a23), s), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

// Many-row path (prefill, M >= 256, K <= AQ_STAGE_MAX_K): one warp per token
// row, 8 rows per CTA, every reduction a warp shuffle or redux (no block
// barrier).  The CTA's 8 rows are staged in shared memory (one bulk copy per
// row, so a whole row is in flight at once) and read there three times: sum
// of squares; normalisation (written back in place) and absmax; codes.  HBM
// reads each row once.  The 8 rows of a CTA share each 128-byte core matrix of
// the tiled code layout, so the CTA writes whole lines.  Same results as
// aq_row_vec: fp64 sum of squares (exact in any order), max, integer sum.
// Dynamic shared memory: 8 * K * 2 bytes (5 CTAs per SM by shared memory at
// K = 2560, 2 at K = 6912).  Requirements as for act_quant_vec_kernel.
constexpr int AQ_STAGE_MAX_K = 14336;  // 8 rows x 2 bytes x K plus the barriers within 227 KB
__global__ void __launch_bounds__(256, 2)
act_quant_rows_kernel(const uint16_t* __restrict__ x, int M, int K, int ldx, const uint16_t* __restrict__ gamma,
                      float eps, int8_t* __restrict__ q, float* __restrict__ row_scale, int32_t* __restrict__ row_sum,
                      uint16_t* __restrict__ normed_out, int T, int Kp) {
  extern __shared__ __align__(16) uint8_t aq_stage_smem[];
  __shared__ uint64_t row_full[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.x * 8 + warp;
  const bool valid = m < M;
  const int KC8 = K >> 3, KP8 = Kp >> 3;
  uint4* row = reinterpret_cast<uint4*>(aq_stage_smem) + (size_t)warp * KC8;
  if (lane == 0) {
    mbar_init(&row_full[warp], 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_trigger();
  pdl_wait();
  if (valid) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&row_full[warp], (uint32_t)(K * 2));
      bulk_g2s(row, x + (size_t)m * ldx, (uint32_t)(K * 2), &row_full[warp]);
    }
    // every lane waits, so each one sees the copied row
    const bool ok = mbar_wait(&row_full[warp], 0, 320);
    if (!__all_sync(0xffffffffu, ok)) {
      // a copy that is still in flight must land before the CTA exits
      if (lane == 0) mbar_wait(&row_full[warp], 0, 321);
      return;
    }
  } else {
    for (int ch = lane; ch < KC8; ch += 32) row[ch] = make_uint4(0, 0, 0, 0);
    __syncwarp();
  }
  const uint4* grow = reinterpret_cast<const uint4*>(gamma);
  uint32_t mx = 0;
  if (gamma != nullptr) {
    double ssp[4] = {0.0, 0.0, 0.0, 0.0};  // four independent chains (exact in any order)
    // the passes are unrolled so that a lane has several chunks' loads and
    // conversions in flight (the kernel is bound by their latency)
#pragma unroll 4
    for (int ch = lane; ch < KC8; ch += 32) aq_sq8(row[ch], ssp);
    double ss = (ssp[0] + ssp[1]) + (ssp[2] + ssp[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float var = __double2float_rn(__ddiv_rn(ss, (double)K));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll 4
    for (int ch = lane; ch < KC8; ch += 32) {
      const uint4 a = aq_norm8(row[ch], grow[ch], r);
      row[ch] = a;
      if (normed_out != nullptr && valid) reinterpret_cast<uint4*>(normed_out + (size_t)m * K)[ch] = a;
      mx = aq_absmax8(mx, a);
    }
  } else {
    for (int ch = lane; ch < KC8; ch += 32) {
      if (normed_out != nullptr && valid) reinterpret_cast<uint4*>(normed_out + (size_t)m * K)[ch] = row[ch];
      mx = aq_absmax8(mx, row[ch]);
    }
  }
  if (q == nullptr) return;
  const float amax = fmaxf(aq_warp_absmax(mx), 1e-5f);
  const float s = __fdiv_rn(127.0f, amax);
  int qsum = 0;
  // chunk ch of the row sits at alayout_offset(m, 8 ch); 32 chunks further on
  // (256 codes) it is 16 core-matrix columns = 256 T bytes further on
  int8_t* qp = q + alayout_offset(m, lane * 8, T, Kp);
  const size_t qstep = (size_t)256 * T;
#pragma unroll 4
  for (int ch = lane; ch < KP8; ch += 32, qp += qstep) {  // chunks past K (up to Kp) are written as zeros
    uint2 o = make_uint2(0, 0);
    if (valid && ch < KC8) {
      const uint4 a = row[ch];
      o.x = aq_codes4(a.x, a.y, s);
      o.y = aq_codes4(a.z, a.w, s);
    }
    qsum = __dp4a((int)o.x, 0x01010101, qsum);
    qsum = __dp4a((int)o.y, 0x01010101, qsum);
    *reinterpret_cast<uint2*>(qp) = o;
  }
  qsum = __reduce_add_sync(0xffffffffu, qsum);
  if (lane == 0) {
    row_scale[m] = valid ? s : 1.0f;
    row_sum[m] = qsum;
  }
}

}  // namespace bitnet
