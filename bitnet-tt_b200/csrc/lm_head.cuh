// Greedy-argmax pieces shared by the lm_head kernels.
//
// token[b] = argmax_v logits[b, v] with the smallest index winning ties
// (torch.argmax).  The lm_head kernel leaves one (max, index) pair per CTA and
// token in the workspace; argmax_reduce_kernel reduces them per token, writes
// the token id and advances the sequence's decode position.
#pragma once
#include "common.cuh"
#include "pack.cuh"

namespace bitnet {

struct ArgPair {
  float v;
  int i;
};
__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// grid = B, block = 256.  Reduces the per-CTA (or per-shard) pairs of each
// token; writes the token id (and advances the sequence's position) or, for a
// vocabulary shard, the token's best (value, index + idx_offset) pair.
__global__ void __launch_bounds__(256)
argmax_reduce_kernel(const ArgPair* __restrict__ part, int ntiles, int B, int32_t* __restrict__ out_ids,
                     int32_t* __restrict__ positions, ArgPair* __restrict__ pair_out, int idx_offset) {
  __shared__ float sv[256];
  __shared__ int si[256];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = tid; t < ntiles; t += 256) {
    const ArgPair a = part[(size_t)t * B + b];
    if (arg_better(a.v, a.i, bv, bi)) {
      bv = a.v;
      bi = a.i;
    }
  }
  sv[tid] = bv;
  si[tid] = bi;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s && arg_better(sv[tid + s], si[tid + s], sv[tid], si[tid])) {
      sv[tid] = sv[tid + s];
      si[tid] = si[tid + s];
    }
    __syncthreads();
  }
  if (tid == 0) {
    if (pair_out != nullptr) {
      pair_out[b] = ArgPair{sv[0], si[0] == 0x7fffffff ? si[0] : si[0] + idx_offset};
    } else {
      out_ids[b] = si[0];
      if (positions != nullptr) positions[b] += 1;
    }
  }
}

}  // namespace bitnet
