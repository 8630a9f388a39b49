// Prefill (prompt) path of the attention: RoPE + KV-cache write for all prompt
// positions, then causal GQA attention over the prompt.
//
// rope_append_prefill_kernel: one CTA per token; the same bf16 op-by-op
// half-split RoPE as the decode kernel:
//     out[i]    = bf16(bf16(x[i] * cos_i)    + bf16(-x[i+64] * sin_i))
//     out[i+64] = bf16(bf16(x[i+64] * cos_i) + bf16( x[i]    * sin_i))
// Rotated queries go to q_out [B*P, n_heads*128]; rotated keys and the values
// go to the caches at rows p = 0 .. P-1.  rope_append_prefill_vec_kernel does
// the same with 16-byte accesses, .f32x2 arithmetic and 8 tokens per CTA when
// every pointer is 16-byte aligned.
//
// attention_prefill_kernel: CTA = (query block of 64 tokens, query head, sequence),
// 4 warps of 16 query rows.  Key blocks of 64 up to the diagonal: K and V rows
// arrive by per-lane cp.async into the XOR-swizzled layout of the decode
// kernel (two blocks in flight); S = Q K^T and O += P V run on mma.sync
// m16n8k16 (bf16 in, fp32 accumulate; P as a bf16 hi + lo pair, each a paired
// conversion); online softmax in fp32 and base 2 (the scale carries log2 e, so
// every exponential is exp2f); causal mask key > query.  Three CTAs per SM
// (at most 168 registers).  Each of these steps was measured at 32 x 512,
// 20 / 5 heads on B200: 317 us per launch before, 291 with the paired
// conversions, 269 with three CTAs per SM, 252 with the base-2 softmax (the
// first two bit-identical, the last within the same error against fp32).
#pragma once
#include "attention.cuh"
#include "common.cuh"

namespace bitnet {

constexpr int APF_THREADS = 128;  // 4 warps x 16 query rows
constexpr int APF_QB = 64;        // query rows per CTA
constexpr int APF_KB = 64;        // keys per block
constexpr int APF_KV_BYTES = APF_KB * ATT_D * 2;  // K (or V) of one key block: 16 KB
constexpr int APF_NBUF = 2;
constexpr size_t APF_SMEM = (size_t)APF_NBUF * 2 * APF_KV_BYTES + 64;  // K|V x 2 buffers + 2 mbarriers

struct RopePrefillParams {
  const uint16_t* qkv;  // [tokens, (n_heads + 2 n_kv) * 128]
  int B, P, n_heads, n_kv;
  const int32_t* cu;    // nullable: sequence b owns tokens cu[b] .. cu[b+1]-1 (ragged prompts); else b*P ..
  int rope_len;
  const uint16_t* rope_cos;  // [>= P, 64]
  const uint16_t* rope_sin;
  uint16_t* q_out;     // [B*P, n_heads * 128]
  uint16_t* k_cache;   // [B, n_kv, max_len, 128]
  uint16_t* v_cache;
  int max_len;
};

// grid = B * P (one CTA per prompt token), 256 threads; a thread takes dims
// (d, d + 1) and (d + 64, d + 65) of one head with 4-byte accesses.
__global__ void __launch_bounds__(256) rope_append_prefill_kernel(const RopePrefillParams p) {
  pdl_trigger();
  pdl_wait();
  const int tok = blockIdx.x;
  int pos, b;
  if (p.cu != nullptr) {
    // the sequence holding this token: the last b with cu[b] <= tok
    int lo = 0, hi = p.B;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.cu[mid] <= tok) lo = mid; else hi = mid;
    }
    b = lo;
    pos = tok - p.cu[b];
    if (pos < 0 || tok >= p.cu[b + 1] || pos >= p.max_len || pos >= p.rope_len) {
      if (threadIdx.x == 0) record_error(DEV_ERR_BOUNDS, 330);
      return;
    }
  } else {
    pos = tok % p.P;
    b = tok / p.P;
  }
  const int nh = p.n_heads + p.n_kv;  // heads that get a rotation
  const uint16_t* row = p.qkv + (size_t)tok * (size_t)((p.n_heads + 2 * p.n_kv) * ATT_D);
  const uint32_t* cs = reinterpret_cast<const uint32_t*>(p.rope_cos + (size_t)pos * 64);
  const uint32_t* sn = reinterpret_cast<const uint32_t*>(p.rope_sin + (size_t)pos * 64);
  for (int it = threadIdx.x; it < nh * 32; it += blockDim.x) {
    const int hh = it >> 5, d = (it & 31) * 2;
    const uint32_t x1 = *reinterpret_cast<const uint32_t*>(row + hh * ATT_D + d);
    const uint32_t x2 = *reinterpret_cast<const uint32_t*>(row + hh * ATT_D + 64 + d);
    const uint32_t c2 = cs[d >> 1], s2 = sn[d >> 1];
    uint32_t o1 = 0, o2 = 0;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float a = bf16_bits_to_f32((uint16_t)(x1 >> (16 * e))), bb = bf16_bits_to_f32((uint16_t)(x2 >> (16 * e)));
      const float c = bf16_bits_to_f32((uint16_t)(c2 >> (16 * e))), sv = bf16_bits_to_f32((uint16_t)(s2 >> (16 * e)));
      const uint16_t r1 = f32_to_bf16_bits(round_bf16(__fadd_rn(round_bf16(__fmul_rn(a, c)), round_bf16(__fmul_rn(-bb, sv)))));
      const uint16_t r2 = f32_to_bf16_bits(round_bf16(__fadd_rn(round_bf16(__fmul_rn(bb, c)), round_bf16(__fmul_rn(a, sv)))));
      o1 |= (uint32_t)r1 << (16 * e);
      o2 |= (uint32_t)r2 << (16 * e);
    }
    if (hh < p.n_heads) {
      uint16_t* dst = p.q_out + (size_t)tok * (size_t)(p.n_heads * ATT_D) + hh * ATT_D;
      *reinterpret_cast<uint32_t*>(dst + d) = o1;
      *reinterpret_cast<uint32_t*>(dst + 64 + d) = o2;
    } else {
      const int g = hh - p.n_heads;
      const size_t crow = (((size_t)b * p.n_kv + g) * p.max_len + pos) * ATT_D;
      *reinterpret_cast<uint32_t*>(p.k_cache + crow + d) = o1;
      *reinterpret_cast<uint32_t*>(p.k_cache + crow + 64 + d) = o2;
      const uint16_t* vsrc = row + (size_t)(p.n_heads + p.n_kv + g) * ATT_D;
      *reinterpret_cast<uint32_t*>(p.v_cache + crow + d) = *reinterpret_cast<const uint32_t*>(vsrc + d);
      *reinterpret_cast<uint32_t*>(p.v_cache + crow + 64 + d) = *reinterpret_cast<const uint32_t*>(vsrc + 64 + d);
    }
  }
}

// The same rotation for two dims of each half (packed bf16 pairs x1 = dims
// (d, d+1), x2 = dims (d+64, d+65)): every product and sum as an .f32x2 pair,
// every rounding one paired conversion.  -x2 * sin is (-x2) * sin with the sign
// flipped on the bf16 bits, as the scalar form computes it.  The adds only see
// bf16-rounded operands.
__device__ __forceinline__ void rope_rotate2(uint32_t x1, uint32_t x2, uint32_t c, uint32_t s, uint32_t& o1,
                                             uint32_t& o2) {
  const uint64_t a = f2_from_bf2(x1), b = f2_from_bf2(x2), nb = f2_from_bf2(x2 ^ 0x80008000u);
  const uint64_t cc = f2_from_bf2(c), ss = f2_from_bf2(s);
  o1 = f2_to_bf2(f2_add(f2_from_bf2(f2_to_bf2(f2_mul(a, cc))), f2_from_bf2(f2_to_bf2(f2_mul(nb, ss)))));
  o2 = f2_to_bf2(f2_add(f2_from_bf2(f2_to_bf2(f2_mul(b, cc))), f2_from_bf2(f2_to_bf2(f2_mul(a, ss)))));
}

// 16-byte form of rope_append_prefill_kernel (every pointer 16-byte aligned):
// a CTA takes RPF_TOK tokens; a work item is 8 dims of both halves of one
// rotated head (query or key; 8 items a head) or 8 dims of one value head (16
// items a head), so each access moves 16 bytes.  Bit-identical results.
constexpr int RPF_TOK = 8;
__global__ void __launch_bounds__(256) rope_append_prefill_vec_kernel(const RopePrefillParams p, int tokens) {
  __shared__ int s_b[RPF_TOK], s_pos[RPF_TOK];
  pdl_trigger();
  pdl_wait();
  const int tok0 = blockIdx.x * RPF_TOK;
  if (threadIdx.x < RPF_TOK) {
    const int tok = tok0 + threadIdx.x;
    int b = -1, pos = 0;
    if (tok < tokens) {
      if (p.cu != nullptr) {
        int lo = 0, hi = p.B;
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (p.cu[mid] <= tok) lo = mid; else hi = mid;
        }
        pos = tok - p.cu[lo];
        if (pos < 0 || tok >= p.cu[lo + 1] || pos >= p.max_len || pos >= p.rope_len)
          record_error(DEV_ERR_BOUNDS, 330);
        else
          b = lo;
      } else {
        pos = tok % p.P;
        b = tok / p.P;
      }
    }
    s_b[threadIdx.x] = b;
    s_pos[threadIdx.x] = pos;
  }
  __syncthreads();
  const int rot_items = (p.n_heads + p.n_kv) * 8, per_tok = rot_items + p.n_kv * 16;
  const size_t row_elems = (size_t)(p.n_heads + 2 * p.n_kv) * ATT_D;
  for (int it = threadIdx.x; it < RPF_TOK * per_tok; it += blockDim.x) {
    const int t = it / per_tok, r = it - t * per_tok;
    const int b = s_b[t];
    if (b < 0) continue;
    const int tok = tok0 + t, pos = s_pos[t];
    const uint16_t* row = p.qkv + (size_t)tok * row_elems;
    if (r < rot_items) {
      const int hh = r >> 3, d = (r & 7) * 8;
      const uint4 x1 = *reinterpret_cast<const uint4*>(row + hh * ATT_D + d);
      const uint4 x2 = *reinterpret_cast<const uint4*>(row + hh * ATT_D + 64 + d);
      const uint4 c = *reinterpret_cast<const uint4*>(p.rope_cos + (size_t)pos * 64 + d);
      const uint4 s = *reinterpret_cast<const uint4*>(p.rope_sin + (size_t)pos * 64 + d);
      uint4 o1, o2;
      rope_rotate2(x1.x, x2.x, c.x, s.x, o1.x, o2.x);
      rope_rotate2(x1.y, x2.y, c.y, s.y, o1.y, o2.y);
      rope_rotate2(x1.z, x2.z, c.z, s.z, o1.z, o2.z);
      rope_rotate2(x1.w, x2.w, c.w, s.w, o1.w, o2.w);
      uint16_t* dst;
      if (hh < p.n_heads)
        dst = p.q_out + (size_t)tok * (size_t)(p.n_heads * ATT_D) + hh * ATT_D;
      else
        dst = p.k_cache + (((size_t)b * p.n_kv + (hh - p.n_heads)) * p.max_len + pos) * ATT_D;
      *reinterpret_cast<uint4*>(dst + d) = o1;
      *reinterpret_cast<uint4*>(dst + 64 + d) = o2;
    } else {
      const int v = r - rot_items, g = v >> 4, c8 = (v & 15) * 8;
      const size_t crow = (((size_t)b * p.n_kv + g) * p.max_len + pos) * ATT_D;
      *reinterpret_cast<uint4*>(p.v_cache + crow + c8) =
          *reinterpret_cast<const uint4*>(row + (size_t)(p.n_heads + p.n_kv + g) * ATT_D + c8);
    }
  }
}

struct AttnPrefillParams {
  const uint16_t* q;  // [B*P, n_heads*128] rotated
  const uint16_t* k_cache;
  const uint16_t* v_cache;
  int B, P, n_heads, n_kv, max_len;  // P: the (longest) prompt length
  float scale;
  uint16_t* out;  // [tokens, n_heads*128]
  const int32_t* cu;  // nullable: token offsets of ragged prompts (sequence b: cu[b] .. cu[b+1]-1)
};

// grid (ceil(P / 64), n_heads, B), 128 threads, APF_SMEM dynamic shared memory.
// mma.sync without volatile: no side effects, so the compiler may interleave
// independent tiles
__device__ __forceinline__ void mma_bf16_16816_nv(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(APF_THREADS, 3) attention_prefill_kernel(const AttnPrefillParams p) {
  extern __shared__ __align__(128) uint8_t smem_apf[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_apf + APF_NBUF * 2 * APF_KV_BYTES);
  pdl_trigger();
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int G = p.n_heads / p.n_kv, g = h / G;
  if (t == 0) {
    for (int i = 0; i < APF_NBUF; ++i) mbar_init(&bars[i], APF_THREADS);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  const int q0 = qb * APF_QB;
  // this sequence's prompt: P tokens from row tok0 of q / out
  int P = p.P;
  size_t tok0 = (size_t)b * p.P;
  if (p.cu != nullptr) {
    tok0 = (size_t)p.cu[b];
    P = p.cu[b + 1] - p.cu[b];
    if (P < 0 || P > p.P || P > p.max_len) {
      if (t == 0 && qb == 0 && h == 0) record_error(DEV_ERR_BOUNDS, 331);
      return;
    }
  }
  if (q0 >= P) return;  // CTA-uniform; nothing issued yet
  const int qend = min(P, q0 + APF_QB);               // query rows of the CTA: [q0, qend)
  const int nkb = (qend - 1) / APF_KB + 1;           // key blocks 0 .. the one holding the last query
  const size_t crow0 = ((size_t)b * p.n_kv + g) * p.max_len;
  const uint16_t* kc = p.k_cache + crow0 * ATT_D;
  const uint16_t* vc = p.v_cache + crow0 * ATT_D;

  // every thread copies 2 x 64 rows x 16 chunks / 128 = 16 chunks of 16 B per block
  auto issue = [&](int kb) {
    const int k0 = kb * APF_KB;
    const uint32_t base = smem_u32(smem_apf + (size_t)(kb % APF_NBUF) * 2 * APF_KV_BYTES);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int q = t + APF_THREADS * j;  // 0 .. 2047
      const int tensor = q >> 10, row = (q >> 4) & 63, c = q & 15;
      const bool in = k0 + row < P;
      const uint16_t* src = (tensor ? vc : kc) + (size_t)(k0 + (in ? row : 0)) * ATT_D + c * 8;
      cp_async16_zfill(base + tensor * APF_KV_BYTES + att_swz(row, c), src, in ? 16u : 0u);
    }
    cp_async_arrive_noinc(&bars[kb % APF_NBUF]);
  };
  for (int kb = 0; kb < min(nkb, APF_NBUF); ++kb) issue(kb);

  // query fragments: rows q0 + 16 warp + (lane / 4) (+ 8), dims 16 ks + 2 (lane % 4) (+ 8)
  const int qr = lane >> 2, qc = 2 * (lane & 3);
  const int row_a = q0 + warp * 16 + qr, row_b = row_a + 8;
  uint32_t qa[8][4];
  {
    const uint16_t* qa_row = p.q + (tok0 + min(row_a, P - 1)) * (size_t)(p.n_heads * ATT_D) + h * ATT_D;
    const uint16_t* qb_row = p.q + (tok0 + min(row_b, P - 1)) * (size_t)(p.n_heads * ATT_D) + h * ATT_D;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = *reinterpret_cast<const uint32_t*>(qa_row + 16 * ks + qc);
      qa[ks][1] = *reinterpret_cast<const uint32_t*>(qb_row + 16 * ks + qc);
      qa[ks][2] = *reinterpret_cast<const uint32_t*>(qa_row + 16 * ks + 8 + qc);
      qa[ks][3] = *reinterpret_cast<const uint32_t*>(qb_row + 16 * ks + 8 + qc);
    }
  }
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[16][4];  // O [16 rows x 128 dims]: n-tile j = dims 8j .. 8j+7
#pragma unroll
  for (int j = 0; j < 16; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  const int mi = lane >> 3, mr = lane & 7;
  const float sl2 = p.scale * 1.4426950408889634f;  // softmax in base 2
  bool ok = true;
  int done = 0;
  for (int kb = 0; kb < nkb; ++kb) {
    ok = mbar_wait(&bars[kb % APF_NBUF], (uint32_t)((kb / APF_NBUF) & 1), 310);
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    const uint32_t kbase = smem_u32(smem_apf + (size_t)(kb % APF_NBUF) * 2 * APF_KV_BYTES);
    const uint32_t vbase = kbase + APF_KV_BYTES;
    const int k0 = kb * APF_KB;
    // S [16 rows x 64 keys]: 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles: keys 16 np .. 16 np + 15
        const int key = np * 16 + (mi >> 1) * 8 + mr;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + att_swz(key, 2 * ks + (mi & 1)), b0, b1, b2, b3);
        mma_bf16_16816_nv(s[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_bf16_16816_nv(s[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
    }
    // mask, scale, online softmax for rows row_a (e 0, 1) and row_b (e 2, 3)
    float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int kk = k0 + 8 * n + qc;
      s[n][0] = (kk <= row_a && kk < P) ? s[n][0] * sl2 : -INFINITY;
      s[n][1] = (kk + 1 <= row_a && kk + 1 < P) ? s[n][1] * sl2 : -INFINITY;
      s[n][2] = (kk <= row_b && kk < P) ? s[n][2] * sl2 : -INFINITY;
      s[n][3] = (kk + 1 <= row_b && kk + 1 < P) ? s[n][3] * sl2 : -INFINITY;
      mxa = fmaxf(mxa, fmaxf(s[n][0], s[n][1]));
      mxb = fmaxf(mxb, fmaxf(s[n][2], s[n][3]));
    }
    mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
    mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
    mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
    mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
    const float mna = fmaxf(m_a, mxa), mnb = fmaxf(m_b, mxb);
    // a row whose keys are all masked so far keeps max -inf: use 0 as the reference
    const float ra = mna == -INFINITY ? 0.f : mna, rb = mnb == -INFINITY ? 0.f : mnb;
    const float ca = exp2f(m_a - ra), cb = exp2f(m_b - rb);
    float sa = 0.f, sb = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = exp2f(s[n][0] - ra);
      s[n][1] = exp2f(s[n][1] - ra);
      s[n][2] = exp2f(s[n][2] - rb);
      s[n][3] = exp2f(s[n][3] - rb);
      sa += s[n][0] + s[n][1];
      sb += s[n][2] + s[n][3];
    }
    sa += __shfl_xor_sync(0xffffffffu, sa, 1);
    sa += __shfl_xor_sync(0xffffffffu, sa, 2);
    sb += __shfl_xor_sync(0xffffffffu, sb, 1);
    sb += __shfl_xor_sync(0xffffffffu, sb, 2);
    l_a = l_a * ca + sa;
    l_b = l_b * cb + sb;
    m_a = mna;
    m_b = mnb;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= ca;
      o[j][1] *= ca;
      o[j][2] *= cb;
      o[j][3] *= cb;
    }
    // O += P V: P (A operand, rows = queries, k = keys) from the S fragments as
    // bf16 hi + lo; V via ldmatrix.trans.  k-step kt = keys 16 kt .. 16 kt + 15.
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
      const float src8[8] = {s[2 * kt][0], s[2 * kt][1], s[2 * kt][2], s[2 * kt][3],
                             s[2 * kt + 1][0], s[2 * kt + 1][1], s[2 * kt + 1][2], s[2 * kt + 1][3]};
      // hi = bf16(p), lo = bf16(p - hi), two values per conversion
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 hv = __floats2bfloat162_rn(src8[2 * e], src8[2 * e + 1]);
        hw[e] = *reinterpret_cast<const uint32_t*>(&hv);
        const __nv_bfloat162 lv = __floats2bfloat162_rn(__fsub_rn(src8[2 * e], __uint_as_float(hw[e] << 16)),
                                                        __fsub_rn(src8[2 * e + 1], __uint_as_float(hw[e] & 0xFFFF0000u)));
        lw[e] = *reinterpret_cast<const uint32_t*>(&lv);
      }
      // a0: (row a, keys 16kt + qc..), a1: (row b, same), a2: (row a, keys + 8), a3: (row b, keys + 8)
      const uint32_t ha0 = hw[0], ha1 = hw[1], ha2 = hw[2], ha3 = hw[3];
      const uint32_t la0 = lw[0], la1 = lw[1], la2 = lw[2], la3 = lw[3];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {  // pairs of dim tiles: dims 16 jj .. 16 jj + 15
        // transposed matrices: (keys 16kt..+7, chunk 2jj), (keys 16kt+8..+15, 2jj), (keys 16kt..+7, 2jj+1), (.., 2jj+1)
        const int key = kt * 16 + (mi & 1) * 8 + mr;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + att_swz(key, 2 * jj + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16_16816_nv(o[2 * jj], ha0, ha1, ha2, ha3, b0, b1);
        mma_bf16_16816_nv(o[2 * jj + 1], ha0, ha1, ha2, ha3, b2, b3);
        mma_bf16_16816_nv(o[2 * jj], la0, la1, la2, la3, b0, b1);
        mma_bf16_16816_nv(o[2 * jj + 1], la0, la1, la2, la3, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with the buffer before it is refilled
    done = kb + 1;
    if (kb + APF_NBUF < nkb) issue(kb + APF_NBUF);
  }
  for (int kb = done; kb < min(nkb, done + APF_NBUF); ++kb) mbar_wait(&bars[kb % APF_NBUF], (uint32_t)((kb / APF_NBUF) & 1), 311);
  if (!ok) return;
  // normalise and write rows row_a / row_b, dims 8 j + qc, + 1
  const float ia = l_a > 0.f ? 1.f / l_a : 0.f, ib = l_b > 0.f ? 1.f / l_b : 0.f;
  uint16_t* oa = p.out + (tok0 + row_a) * (size_t)(p.n_heads * ATT_D) + h * ATT_D;
  uint16_t* ob = p.out + (tok0 + row_b) * (size_t)(p.n_heads * ATT_D) + h * ATT_D;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (row_a < P)
      *reinterpret_cast<uint32_t*>(oa + 8 * j + qc) = pack_bf16x2(o[j][0] * ia, o[j][1] * ia);
    if (row_b < P)
      *reinterpret_cast<uint32_t*>(ob + 8 * j + qc) = pack_bf16x2(o[j][2] * ib, o[j][3] * ib);
  }
}

}  // namespace bitnet
