/*
 * bitnet_b200.h -- C ABI of the B200 (sm_100a) packed-ternary BitLinear decode path.
 *
 * All tensor pointers are DEVICE pointers owned by the caller.  No entry point
 * allocates memory, synchronises the device or writes host memory; every launch
 * is ordered on the stream passed in (a cudaStream_t; NULL is the legacy default
 * stream), so all of them can be recorded into a CUDA graph.  Every entry point
 * returns 0 (BITNET_OK) or a negative status; bitnet_status_string() names it.
 * Nothing throws across the ABI.  Calls on distinct streams with distinct
 * output buffers are independent.
 *
 * bf16 tensors are passed as `void*` and are IEEE bfloat16 (torch.bfloat16).
 *
 * The reference project drives this path through ttnn (Tenstorrent) ops; each
 * declaration below names the reference interface it replaces
 * (path:line inside deveworld/bitnet-tt).
 */
#ifndef BITNET_B200_H
#define BITNET_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* bitnet_stream_t; /* cudaStream_t */

/* ---- status codes ------------------------------------------------------ */
#define BITNET_OK 0
#define BITNET_ERR_INVALID_ARGUMENT (-1) /* shape, null pointer or option out of range   */
#define BITNET_ERR_ALIGNMENT (-2)        /* a pointer is not aligned as documented          */
#define BITNET_ERR_UNSUPPORTED_DEVICE (-3) /* the current device is not sm_100             */
#define BITNET_ERR_CUDA (-4)             /* a CUDA runtime call (launch, attribute) failed  */
#define BITNET_ERR_DEVICE_TIMEOUT (-5)   /* a kernel gave up a bounded wait (see below)     */
#define BITNET_ERR_SCRATCH_LIMIT (-6)    /* problem larger than bitnet_bitlinear_noalloc's static scratch */

/* ---- BitLinear epilogues ------------------------------------------------ */
#define BITNET_EPI_NONE 0          /* y = bf16(acc * w_scale / s_m)                                */
#define BITNET_EPI_RELU2_MUL 1     /* rows in 64-row groups [32 gate | 32 up]: y = relu(g)^2 * u   */
#define BITNET_EPI_RESIDUAL_ADD 2  /* y = bf16(residual + bf16(acc * w_scale / s_m))               */

/* ---- BitLinear execution paths ------------------------------------------ */
#define BITNET_PATH_AUTO 0    /* SIMT below the ridge batch, tcgen05 above it               */
#define BITNET_PATH_SIMT 1    /* CUDA-core unpack + dp4a, HBM-bound for M <= 4              */
#define BITNET_PATH_TCGEN05 2 /* tcgen05 kind::i8 MMA, weights unpacked into TMEM        */

#define BITNET_MAX_SEGMENTS 4
/* Per-tensor weight scales of a fused projection (QKV has 3 segments, a plain
 * projection 1).  Segment i covers output rows [end[i-1], end[i]).  For the
 * RELU2_MUL epilogue scale[0] is the gate scale and scale[1] the up scale. */
typedef struct {
  int32_t count;
  int32_t end[BITNET_MAX_SEGMENTS];
  float scale[BITNET_MAX_SEGMENTS];
} bitnet_segments_t;

/* ---- library information -------------------------------------------------- */
int bitnet_abi_version(void);
const char* bitnet_status_string(int status);
/* Reads and clears the library's device status word (set by a kernel that gave
 * up a bounded wait).  Synchronises the current device.  *site (nullable)
 * receives the id of the wait that gave up. */
int bitnet_last_device_status(int* site);
/* Text of the last CUDA runtime failure reported as BITNET_ERR_CUDA on the
 * calling thread (the failing call, cudaGetErrorString, code). */
const char* bitnet_last_cuda_error(void);
/* Self-test of the bounded waits (no reference counterpart): launches one CTA
 * whose mbarrier wait can never complete (nothing arrives on it).  The wait
 * gives up after limit_cycles SM clocks (1 .. 2^31), records
 * BITNET_ERR_DEVICE_TIMEOUT with site 900 in the device status word, and the
 * kernel returns -- how every wait of the library's kernels ends when it runs
 * out, shown without faulting or hanging the GPU.  The context stays usable. */
int bitnet_selftest_bounded_wait(long long limit_cycles, bitnet_stream_t stream);

/* ---- process-wide launch options (no reference counterpart: ttnn chooses
 * program configs internally) -------------------------------------------- */
/* Launch kernels with programmatic dependent launch (default 1). */
int bitnet_set_pdl(int enable);
/* Force the K split (cluster size, 1..8) of the tcgen05 path; 0 = automatic. */
int bitnet_set_tc_split(int split);
/* BITNET_PATH_AUTO uses the SIMT path for M <= m (0..8, default 4). */
int bitnet_set_simt_max_m(int m);

/* ---- sizes of caller-owned buffers ------------------------------------------ */
/* Bytes of the device weight layout for an [N, K] ternary matrix
 * (rows padded to 128, K padded to 64, 2 bits per weight). */
size_t bitnet_packed_weight_bytes(int N, int K);
/* Bytes of the int8 activation buffer for M tokens x K features (token tiles of
 * at most 256 rows, K padded to 64).  row_scale / row_sum need bitnet_act_rows(M)
 * entries each. */
size_t bitnet_act_bytes(int M, int K);
int bitnet_act_rows(int M);

/* ---- weight packing (load time) -------------------------------------------
 * Replaces the packed_ternary branch of Linear.load_weights /
 * load_pretransposed_weight (src/bitnet_tt/layers/bitlinear.py:211-251, 269-298),
 * which packs BFP2_b tiles for Tensix.  Input: int8 ternary codes W_q [N, K]
 * row-major (values -1, 0, +1; anything else is treated as 0). */
int bitnet_pack_ternary(const int8_t* w_q, int N, int K, uint8_t* w_packed, bitnet_stream_t stream);
/* Same, from the repo's canonical 2-bit format produced by
 * pack_ternary_weights (src/bitnet_tt/utils/quantization.py:111-138): the
 * row-major [N, K] matrix flattened, 4 codes (w + 1) per byte, MSB first. */
int bitnet_pack_from_canonical(const uint8_t* canonical, int N, int K, uint8_t* w_packed,
                               bitnet_stream_t stream);
/* Same, from the reference's Tensix tile format (src/bitnet_tt/kernels/pack.py:101-155
 * pack_ternary_tilized, read by src/bitnet_tt/kernels/device/reader_ternary_in1.cpp:44-55,
 * 86-113; the tiled ternary weight the packed_ternary Linear.load_weights stores,
 * src/bitnet_tt/layers/bitlinear.py:211-251): W^T [K, N] in 32 x 32 tiles, tile
 * (kt, nt) at index kt * ceil(N/32) + nt, 256 bytes each; inside a tile the four
 * 16 x 16 faces TL, TR, BL, BR, each row major, 4 codes per byte MSB first,
 * codes 0b00 = 0, 0b01 = +1, 0b10 = -1 (0b11 reads as 0).  `tiles` holds
 * bitnet_tilized_weight_bytes(N, K) bytes (K and N padded to 32 with zeros). */
size_t bitnet_tilized_weight_bytes(int N, int K);
int bitnet_pack_from_tilized(const uint8_t* tiles, int N, int K, uint8_t* w_packed, bitnet_stream_t stream);

/* ---- fused RMSNorm + per-token int8 absmax quantisation --------------------
 * Replaces ttnn.rms_norm (src/bitnet_tt/layers/bitlinear.py:433-461) feeding
 * the activation quantiser activation_quant_absmax
 * (src/bitnet_tt/utils/quantization.py:60-91).
 * x: bf16 [M, K] with row stride ldx elements.  gamma: bf16 [K] or NULL (no norm).
 * q: int8 activation buffer (bitnet_act_bytes), row_scale[m] = 127 / absmax,
 * row_sum[m] = sum_k q[m, k].  normed_out (nullable): the bf16 normalised rows
 * [M, K] (contiguous).  q, row_scale and row_sum may all be NULL when only
 * normed_out is wanted (plain RMSNorm). */
int bitnet_act_quant(const void* x, int M, int K, int ldx, const void* gamma, float eps, int8_t* q,
                     float* row_scale, int32_t* row_sum, void* normed_out, bitnet_stream_t stream);

/* ---- BitLinear from quantised activations -----------------------------------
 * Replaces ttnn.experimental.ternary_matmul(x, w, use_packed_ternary=True, ...)
 * plus the post-scale of Linear.__call__ (src/bitnet_tt/layers/bitlinear.py:309-353,
 * op call 336-341, scale 351-352) and the fused-projection epilogues of
 * FeedForward.__call__ (src/bitnet_tt/layers/ffn.py:140-170) and the residual
 * adds of the decode step (src/bitnet_tt/inference/generator_batch32.py:749, 756).
 * acc[m, n] = sum_k q[m, k] * W[n, k] (int32, exact); y = bf16(acc * (scale_seg(n) / row_scale[m])).
 * y: bf16 [M, N] ([M, N/2] for RELU2_MUL).  residual: bf16 [M, N] for RESIDUAL_ADD
 * (may alias y).  acc_out (nullable): int32 [M, N] accumulators, for parity checks. */
int bitnet_bitlinear_q(const int8_t* q, const float* row_scale, const int32_t* row_sum, int M, int K,
                       const uint8_t* w_packed, int N, const bitnet_segments_t* segments, int epilogue,
                       const void* residual, void* y, int32_t* acc_out, int path, bitnet_stream_t stream);

/* ---- fused BitLinear (norm + quant + ternary matmul + epilogue) --------------
 * bitnet_act_quant followed by bitnet_bitlinear_q; q_ws / scale_ws / sum_ws are
 * the caller's activation buffers (bitnet_act_bytes / bitnet_act_rows).
 * Replaces the fused-norm ternary_matmul call of the decode step
 * (src/bitnet_tt/inference/generator_batch32.py:718-727). */
int bitnet_bitlinear(const void* x, int M, int K, const void* gamma, float eps, const uint8_t* w_packed,
                     int N, const bitnet_segments_t* segments, int epilogue, const void* residual, void* y,
                     int32_t* acc_out, int8_t* q_ws, float* scale_ws, int32_t* sum_ws, int path,
                     bitnet_stream_t stream);

/* ---- fused BitLinear without caller-provided scratch ------------------------
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory where they call -- an FFI host (cgo, JNI, a C plugin)
 * that holds no CUDA allocator, or code that runs where allocation is not
 * allowed.  Same arguments and results as bitnet_bitlinear, minus q_ws /
 * scale_ws / sum_ws: the int8 activations, row scales and row sums live in a
 * static device array of the library (BITNET_NOALLOC_MAX_ACT_BYTES bytes plus
 * 2 KB), held by every GPU that loads the library until the process exits.
 * Calls with bitnet_act_rows(M) > BITNET_NOALLOC_MAX_ROWS or
 * bitnet_act_rows(M) * round_up(K, 64) > BITNET_NOALLOC_MAX_ACT_BYTES return
 * BITNET_ERR_SCRATCH_LIMIT.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) and should therefore come before any
 * stream capture on that device.  Every call shares the one array, so calls
 * whose kernels overlap on the GPU (other streams, other host threads) race;
 * serialise them.  No allocation happens inside. */
#define BITNET_NOALLOC_MAX_ROWS 256
#define BITNET_NOALLOC_MAX_ACT_BYTES (1u << 20)
int bitnet_bitlinear_noalloc(const void* x, int M, int K, const void* gamma, float eps, const uint8_t* w_packed,
                             int N, const bitnet_segments_t* segments, int epilogue, const void* residual, void* y,
                             int32_t* acc_out, int path, bitnet_stream_t stream);

/* ---- GQA decode attention with fused RoPE and KV append --------------------
 * Replaces nlp_create_qkv_heads_decode + rotary_embedding_llama +
 * paged_update_cache + scaled_dot_product_attention_decode +
 * nlp_concat_heads_decode (src/bitnet_tt/layers/attention.py:1040-1262; the
 * SDPA decode's chunked grid, attention.py:670-708, becomes a split of each
 * context over up to ceil(max_ctx / 256) CTAs with an in-kernel merge; the
 * count per (sequence, KV head) minimises waves x unit length over the GPU,
 * so many long contexts run one CTA each and a few spread wide).
 * qkv: bf16 [B, (n_heads + 2*n_kv_heads) * head_dim] (Q | K | V, already scaled),
 * 4-byte aligned.
 * positions: int32 [B], the position of the token being decoded per sequence.
 * rope_cos / rope_sin: bf16 [rope_len, head_dim/2] (HF half-split convention).
 * k_cache / v_cache: bf16 [B, n_kv_heads, max_len, head_dim]; row `positions[b]`
 * is overwritten with the rotated K / V of this token.
 * max_ctx: an upper bound on positions[b] + 1 for this call (0 = min(max_len,
 * rope_len)); it sets the number of context splits, so a tight bound keeps the
 * grid small.  A position at or above it is a device bounds error.
 * workspace: bitnet_gqa_decode_workspace_bytes(B, n_heads, n_kv_heads, max_ctx)
 * bytes, 16-byte aligned, ZEROED before its first use (the kernel leaves it
 * zeroed); may be NULL when that size is 0 (one CTA per (sequence, KV head):
 * max_ctx <= 256, or enough sequences to fill the GPU).
 * out: bf16 [B, n_heads * head_dim].  head_dim must be 128. */
size_t bitnet_gqa_decode_workspace_bytes(int B, int n_heads, int n_kv_heads, int max_ctx);
int bitnet_gqa_decode_attention(const void* qkv, int B, int n_heads, int n_kv_heads, int head_dim,
                                const int32_t* positions, const void* rope_cos, const void* rope_sin,
                                int rope_len, void* k_cache, void* v_cache, int max_len, int max_ctx, float scale,
                                void* workspace, size_t workspace_bytes, void* out, bitnet_stream_t stream);

/* ---- persistent decode of every layer -----------------------------------
 * One launch runs all transformer layers of a decode step (the per-layer
 * sequence of src/bitnet_tt/model/transformer.py:59-120 and
 * inference/generator_batch32.py:656-811, _decode_step_batch32, up to the
 * final norm): for each layer the input_layernorm act-quant, the fused QKV
 * BitLinear, RoPE + KV append + GQA attention, attn_sub_norm act-quant, o_proj
 * + residual, post_attention_layernorm act-quant, gate_up + ReLU^2 * up,
 * ffn_sub_norm act-quant, down + residual.  Results are bit-identical to the
 * same sequence of the per-operation entry points above.  No counterpart in
 * the reference (there, each operation is its own device program inside the
 * captured trace).
 * Requirements: batch <= 32, head_dim 128, n_heads / n_kv_heads in {1,2,4,8},
 * hidden, intermediate and n_heads*128 multiples of 8 and at most 8192,
 * 16-byte aligned buffers; attention arguments as in
 * bitnet_gqa_decode_attention (the caches come from the layers). */
typedef struct {
  const uint8_t* w_qkv;         /* packed [(n_heads + 2 n_kv) * 128, hidden], segments q | k | v */
  const uint8_t* w_o;           /* packed [hidden, n_heads * 128] */
  const uint8_t* w_gate_up;     /* packed [2 * intermediate, hidden], 64-row groups [32 gate | 32 up] */
  const uint8_t* w_down;        /* packed [hidden, intermediate] */
  bitnet_segments_t seg_qkv, seg_o, seg_gate_up, seg_down; /* per-tensor weight scales */
  const void* input_layernorm;  /* bf16 [hidden] */
  const void* attn_sub_norm;    /* bf16 [n_heads * 128] */
  const void* post_attention_layernorm; /* bf16 [hidden] */
  const void* ffn_sub_norm;     /* bf16 [intermediate] */
  void* k_cache;                /* bf16 [batch, n_kv, max_len, 128] */
  void* v_cache;
} bitnet_decode_layer_t;

typedef struct {
  int num_layers, batch, hidden, intermediate, n_heads, n_kv_heads, head_dim;
  float eps;
  const bitnet_decode_layer_t* layers; /* host array [num_layers]; copied at plan creation */
  void* hidden_state;           /* bf16 [batch, hidden]: the embeddings in, the last layer's output out */
  void* qkv;                    /* bf16 [batch, (n_heads + 2 n_kv) * 128] scratch */
  void* attn;                   /* bf16 [batch, n_heads * 128] scratch */
  void* mid;                    /* bf16 [batch, intermediate] scratch */
  const int32_t* positions;
  const void* rope_cos;
  const void* rope_sin;
  int rope_len, max_len, max_ctx;
  void* attn_workspace;         /* as for bitnet_gqa_decode_attention (zeroed once) */
  size_t attn_workspace_bytes;
  int splits[4];                /* K splits of the qkv, o, gate_up and down BitLinears (0 = automatic) */
} bitnet_decode_desc_t;

typedef struct bitnet_decode_plan bitnet_decode_plan_t;
/* Validates the description, chooses the work split and allocates the plan's
 * device scratch (activation codes, split-K partial sums, grid barrier). */
int bitnet_decode_plan_create(const bitnet_decode_desc_t* desc, bitnet_decode_plan_t** plan);
/* Enqueues one pass over all layers on `stream` (capturable in a CUDA graph). */
int bitnet_decode_plan_run(bitnet_decode_plan_t* plan, bitnet_stream_t stream);
int bitnet_decode_plan_destroy(bitnet_decode_plan_t* plan);

/* ---- prefill (prompt) attention ------------------------------------------
 * Replaces the prefill branch of the attention (src/bitnet_tt/layers/
 * attention.py:1348-1507 and model/bitnet.py:217-313: all prompt tokens of a
 * batch in one pass).
 * bitnet_rope_append_prefill: qkv bf16 [B*P, (n_heads + 2 n_kv) * 128] (token
 * b*P + p at position p) -> rotated queries q_out bf16 [B*P, n_heads * 128];
 * rotated keys and the values written to cache rows 0 .. P-1.
 * bitnet_attention_prefill: causal GQA attention of every prompt token over
 * the cache rows 0 .. its position; out bf16 [B*P, n_heads * 128]. */
int bitnet_rope_append_prefill(const void* qkv, int B, int P, int n_heads, int n_kv_heads, int head_dim,
                               const void* rope_cos, const void* rope_sin, int rope_len, void* q_out, void* k_cache,
                               void* v_cache, int max_len, bitnet_stream_t stream);
int bitnet_attention_prefill(const void* q, const void* k_cache, const void* v_cache, int B, int P, int n_heads,
                             int n_kv_heads, int head_dim, int max_len, float scale, void* out,
                             bitnet_stream_t stream);
/* Ragged prompts: sequence b owns the packed token rows cu_seqlens[b] ..
 * cu_seqlens[b+1]-1 (int32 [B+1] on the device, cu_seqlens[0] = 0,
 * cu_seqlens[B] = total_tokens), at positions 0 .. its length - 1; max_seqlen
 * bounds every length (it sizes the grid).  A length beyond max_seqlen /
 * max_len / rope_len is a device bounds error (bitnet_last_device_status). */
int bitnet_rope_append_prefill_varlen(const void* qkv, int B, const int32_t* cu_seqlens, int total_tokens,
                                      int max_seqlen, int n_heads, int n_kv_heads, int head_dim,
                                      const void* rope_cos, const void* rope_sin, int rope_len, void* q_out,
                                      void* k_cache, void* v_cache, int max_len, bitnet_stream_t stream);
int bitnet_attention_prefill_varlen(const void* q, const void* k_cache, const void* v_cache, int B,
                                    const int32_t* cu_seqlens, int max_seqlen, int n_heads, int n_kv_heads,
                                    int head_dim, int max_len, float scale, void* out, bitnet_stream_t stream);

/* ---- lm_head / embedding table -------------------------------------------
 * The tied embedding / lm_head matrix (src/bitnet_tt/utils/weights.py:236-246)
 * is stored once, in a tiled layout read by both the lm_head and the gather. */
size_t bitnet_lm_head_bytes(int V, int K);
int bitnet_pack_lm_head(const void* w, int V, int K, void* w_tiled, bitnet_stream_t stream);
/* Embedding lookup (src/bitnet_tt/layers/embedding.py:14-70 and the host-side
 * embed copy of src/bitnet_tt/inference/generator_batch32.py:981-1003):
 * out[b, :] = W[ids[b], :], bf16 [B, K]. */
int bitnet_embed_gather(const int32_t* ids, int B, const void* w_tiled, int V, int K, void* out,
                        bitnet_stream_t stream);

/* ---- lm_head with fused greedy argmax ---------------------------------------
 * Replaces the lm_head matmul chunks + ttnn.argmax of the decode step
 * (src/bitnet_tt/inference/generator_batch32.py:768-811, 1170-1174).
 * h: bf16 [B, K] (already final-normed).  out_ids[b] = argmax_v bf16(h[b] . W[v])
 * (first index on ties); B <= 256.  workspace: bitnet_argmax_workspace_bytes(B, K, V)
 * bytes, 256-byte aligned (per-CTA partial maxima + the hidden states re-tiled
 * for the tensor cores).
 * logits_out (nullable): bf16 [B, V].  advance_positions (nullable): int32 [B],
 * incremented by one after the ids are written (the next decode position). */
size_t bitnet_argmax_workspace_bytes(int B, int K, int V);
int bitnet_lm_head_argmax(const void* h, int B, int K, const void* w_tiled, int V, void* workspace,
                          int32_t* out_ids, void* logits_out, int32_t* advance_positions,
                          bitnet_stream_t stream);

/* ---- vocabulary-sharded lm_head (multi-GPU, batch split) -------------------
 * No counterpart in the reference (its lm_head runs on one device).  Rank r of
 * N holds rows [vocab_offset, vocab_offset + V_shard) of the tiled table
 * (bitnet_pack_lm_head of that slice).  A step gathers every rank's normed
 * hidden rows (B = N x batch), runs the shard, gathers the per-row pairs of
 * all ranks and merges them:
 *   bitnet_lm_head_argmax_shard: pairs_out[b] = (best bf16 logit, global row
 *     index) of row b over the shard; ties keep the smaller index.  8-byte
 *     aligned [B] array of {float value; int32 index}.  Workspace as for
 *     bitnet_lm_head_argmax (bitnet_argmax_workspace_bytes(B, K, V_shard)).
 *   bitnet_argmax_merge_pairs: pairs [nshard][B] -> out_ids[b] = index of the
 *     best pair (larger value, then smaller index); advances positions if
 *     given.  The result equals bitnet_lm_head_argmax over the whole table. */
int bitnet_lm_head_argmax_shard(const void* h, int B, int K, const void* w_tiled_shard, int V_shard,
                                int vocab_offset, void* workspace, void* pairs_out, bitnet_stream_t stream);
int bitnet_argmax_merge_pairs(const void* pairs, int nshard, int B, int32_t* out_ids, int32_t* advance_positions,
                              bitnet_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BITNET_B200_H */
