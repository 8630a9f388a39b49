// Load-time re-layout of ternary weights into the device weight layout.
//
// Device layout (2 bits per weight, rows padded to 128, K padded to 64):
//   [N/128 row blocks][K/64 chunks][128 rows][16 bytes]
// A 16-byte cell holds 64 consecutive K positions of one row as four 32-bit
// words; word i covers K offsets 16*i .. 16*i+15, and inside a word the code of
// element e = 4*j + b (code = w + 1 in {0,1,2}) sits at bits [8*b + 2*j, +2), so
// that (word >> 2j) & 0x03030303 yields four int8 codes for K offsets 4j..4j+3.
// A warp reading 16 bytes per lane for 32 consecutive rows touches 512
// contiguous bytes, and one (row block, K range) slice is contiguous, so a CTA
// moves its whole slice with a single bulk copy.
#pragma once
#include "common.cuh"

namespace bitnet {

// One thread per 32-bit output word.
__global__ void pack_ternary_kernel(const int8_t* __restrict__ w_q, int N, int K, int Npad, int KC,
                                    uint32_t* __restrict__ out) {
  const size_t total = (size_t)Npad * KC * 4;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    // idx enumerates words in memory order: ((nb*KC + kc)*128 + r)*4 + wi
    const int wi = (int)(idx & 3);
    const size_t cell = idx >> 2;
    const int r = (int)(cell & 127);
    const size_t blk = cell >> 7;
    const int kc = (int)(blk % KC);
    const int nb = (int)(blk / KC);
    const int n = nb * 128 + r;
    const int kbase = kc * 64 + wi * 16;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int k = kbase + e;
      int v = 0;
      if (n < N && k < K) v = w_q[(size_t)n * K + k];
      const uint32_t code = (v == 1) ? 2u : (v == -1 ? 0u : 1u);
      const int j = e >> 2, b = e & 3;
      word |= code << (8 * b + 2 * j);
    }
    out[idx] = word;
  }
}

// Same output, reading the canonical flat MSB-first 2-bit format
// (byte f/4 of the flattened matrix holds element f at bits 6-2*(f%4)).
__global__ void pack_from_canonical_kernel(const uint8_t* __restrict__ canon, int N, int K, int Npad, int KC,
                                           uint32_t* __restrict__ out) {
  const size_t total = (size_t)Npad * KC * 4;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int wi = (int)(idx & 3);
    const size_t cell = idx >> 2;
    const int r = (int)(cell & 127);
    const size_t blk = cell >> 7;
    const int kc = (int)(blk % KC);
    const int nb = (int)(blk / KC);
    const int n = nb * 128 + r;
    const int kbase = kc * 64 + wi * 16;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int k = kbase + e;
      uint32_t code = 1u;
      if (n < N && k < K) {
        const size_t f = (size_t)n * K + k;
        code = (canon[f >> 2] >> (6 - 2 * (int)(f & 3))) & 3u;
        if (code == 3u) code = 1u;  // not a valid code: treated as a zero weight
      }
      const int j = e >> 2, b = e & 3;
      word |= code << (8 * b + 2 * j);
    }
    out[idx] = word;
  }
}

// Same output, reading the reference's Tensix tile format (kernels/pack.py:101-155,
// consumed by kernels/device/reader_ternary_in1.cpp:44-55, 86-113): the transposed
// matrix W^T [K, N] cut into 32 x 32 tiles, tile (kt, nt) at index kt * Nt + nt
// (Nt = ceil(N / 32)), 256 bytes per tile.  Inside a tile the four 16 x 16 faces
// (top-left, top-right, bottom-left, bottom-right) follow one another, each row
// major; element e of that order sits in byte e / 4 at bits 6 - 2 * (e % 4)
// (MSB first), with the Tensix codes 0b00 = 0, 0b01 = +1, 0b10 = -1 (0b11 is
// reserved and read as 0, as the reference's lookup table does).
__device__ __forceinline__ uint32_t tilized_code(const uint8_t* __restrict__ tiles, int n, int k, int Nt) {
  const int kt = k >> 5, nt = n >> 5, r = k & 31, c = n & 31;
  const int e = ((r >> 4) * 2 + (c >> 4)) * 256 + (r & 15) * 16 + (c & 15);
  const uint32_t t = (tiles[((size_t)kt * Nt + nt) * 256u + (e >> 2)] >> (6 - 2 * (e & 3))) & 3u;
  return t == 1u ? 2u : (t == 2u ? 0u : 1u);  // Tensix code -> device code w + 1
}

__global__ void pack_from_tilized_kernel(const uint8_t* __restrict__ tiles, int N, int K, int Npad, int KC,
                                         uint32_t* __restrict__ out) {
  const int Nt = (N + 31) >> 5;
  const size_t total = (size_t)Npad * KC * 4;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int wi = (int)(idx & 3);
    const size_t cell = idx >> 2;
    const int r = (int)(cell & 127);
    const size_t blk = cell >> 7;
    const int kc = (int)(blk % KC);
    const int nb = (int)(blk / KC);
    const int n = nb * 128 + r;
    const int kbase = kc * 64 + wi * 16;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int k = kbase + e;
      const uint32_t code = (n < N && k < K) ? tilized_code(tiles, n, k, Nt) : 1u;
      const int j = e >> 2, b = e & 3;
      word |= code << (8 * b + 2 * j);
    }
    out[idx] = word;
  }
}

// lm_head / embedding table: bf16 [V, K] -> [V/128 tiles][K/8 chunks][128 rows][8 bf16].
// Each (tile, chunk) block is 2 KB of 16 tcgen05 core matrices (8 rows x 16 B).
__global__ void pack_lm_head_kernel(const uint16_t* __restrict__ w, int V, int K, int Vpad, int KC8,
                                    uint4* __restrict__ out) {
  const size_t total = (size_t)Vpad * KC8;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(idx & 127);
    const size_t blk = idx >> 7;
    const int c = (int)(blk % KC8);
    const int vt = (int)(blk / KC8);
    const int v = vt * 128 + r;
    uint16_t e[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = c * 8 + i;
      e[i] = (v < V && k < K) ? w[(size_t)v * K + k] : (uint16_t)0;
    }
    uint4 o;
    o.x = (uint32_t)e[0] | ((uint32_t)e[1] << 16);
    o.y = (uint32_t)e[2] | ((uint32_t)e[3] << 16);
    o.z = (uint32_t)e[4] | ((uint32_t)e[5] << 16);
    o.w = (uint32_t)e[6] | ((uint32_t)e[7] << 16);
    out[idx] = o;
  }
}

__host__ __device__ __forceinline__ size_t lm_layout_offset16(int v, int c8, int KC8) {
  // offset in 16-byte units of row v, K chunk c8 (8 bf16)
  return ((size_t)(v >> 7) * KC8 + c8) * 128u + (size_t)(v & 127);
}

// out[b, :] = table[ids[b], :] (bf16), one thread per 16-byte chunk.
__global__ void embed_gather_kernel(const int32_t* __restrict__ ids, int B, const uint4* __restrict__ table,
                                    int V, int K, int KC8, uint16_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  if (b >= B) return;
  int v = ids[b];
  if (v < 0 || v >= V) {
    record_error(DEV_ERR_BOUNDS, 100);
    v = 0;
  }
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < KC8; c += gridDim.x * blockDim.x) {
    const uint4 val = table[lm_layout_offset16(v, c, KC8)];
    const int k0 = c * 8;
    uint16_t* dst = out + (size_t)b * K + k0;
    if (k0 + 8 <= K && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
      *reinterpret_cast<uint4*>(dst) = val;
    } else {
      const uint16_t e[8] = {(uint16_t)(val.x & 0xFFFF), (uint16_t)(val.x >> 16), (uint16_t)(val.y & 0xFFFF),
                             (uint16_t)(val.y >> 16),    (uint16_t)(val.z & 0xFFFF), (uint16_t)(val.z >> 16),
                             (uint16_t)(val.w & 0xFFFF), (uint16_t)(val.w >> 16)};
      for (int i = 0; i < 8 && k0 + i < K; ++i) dst[i] = e[i];
    }
  }
}

}  // namespace bitnet
