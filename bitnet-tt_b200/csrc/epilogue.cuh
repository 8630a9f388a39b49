// BitLinear epilogue arithmetic shared by the SIMT and tcgen05 paths.
//
// The ternary contraction runs on codes c = w + 1 in {0,1,2}, so the kernels
// accumulate acc' = sum_k c_k q_k = acc + sum_k q_k; the exact ternary
// accumulator is acc = acc' - row_sum[m].  The scale step is fixed as
//   f = w_scale / s_m          (fp32 divide, s_m = 127 / absmax of the token)
//   y = bf16(float(acc) * f)   (fp32 multiply, round to nearest even)
// float(acc) is exact because |acc| <= 128 * K < 2^24 for K <= 131072.
#pragma once
#include "common.cuh"

struct bitnet_segments_dev {
  int count;
  int end[4];
  float scale[4];
};

namespace bitnet {

enum Epilogue : int { EPI_NONE = 0, EPI_RELU2_MUL = 1, EPI_RESIDUAL_ADD = 2 };

__device__ __forceinline__ float seg_scale_of(const bitnet_segments_dev& seg, int n) {
  float s = seg.scale[0];
#pragma unroll
  for (int i = 1; i < 4; ++i)
    if (i < seg.count && n >= seg.end[i - 1]) s = seg.scale[i];
  return s;
}

// float(acc) without the conversion pipe when |acc| < 2^22 (small): the bits
// of 1.5 * 2^23 plus acc are the float 1.5 * 2^23 + acc, and subtracting
// 1.5 * 2^23 is exact.  |acc| <= 127 K, so small holds for K <= 16384.
__device__ __forceinline__ float i2f_exact(int acc, bool small) {
  return small ? __fsub_rn(__int_as_float(acc + 0x4B400000), 12582912.0f) : (float)acc;
}

// bf16(acc * (w_scale / s_m)), returned widened to fp32.
__device__ __forceinline__ float scaled_bf16(int acc, float w_scale, float s_m) {
  const float f = __fdiv_rn(w_scale, s_m);
  return round_bf16(__fmul_rn((float)acc, f));
}

// HF ReLUSquaredActivation(gate) * up in bf16 ops: relu, square (bf16), multiply (bf16).
__device__ __forceinline__ uint16_t relu2_mul_bf16(float g, float u) {
  const float r = g > 0.f ? round_bf16(__fmul_rn(g, g)) : 0.f;
  return f32_to_bf16_bits(__fmul_rn(r, u));
}

__device__ __forceinline__ uint16_t residual_add_bf16(uint16_t res, float v) {
  return f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(res), v));
}

// The same two steps on packed pairs of bf16 values (element 0 in the low
// half): the products and sums as .f32x2, each rounding one paired
// conversion.  Results equal relu2_mul_bf16 / residual_add_bf16 per element.
__device__ __forceinline__ uint32_t relu2_mul_bf2(uint32_t g, uint32_t u) {
  const uint64_t gf = f2_from_bf2(g);
  const uint32_t keep = (__uint_as_float(g << 16) > 0.f ? 0x0000FFFFu : 0u) |
                        (__uint_as_float(g & 0xFFFF0000u) > 0.f ? 0xFFFF0000u : 0u);
  const uint32_t r = f2_to_bf2(f2_mul(gf, gf)) & keep;  // relu(g)^2 rounded; +0 where g <= 0
  return f2_to_bf2(f2_mul(f2_from_bf2(r), f2_from_bf2(u)));
}
__device__ __forceinline__ uint32_t residual_add_bf2(uint32_t res, uint32_t v) {
  return f2_to_bf2(f2_add(f2_from_bf2(res), f2_from_bf2(v)));
}

}  // namespace bitnet
