"""ctypes binding of the C ABI in include/bitnet_b200.h (libbitnet_b200.so).

Only plain pointers, ints and floats cross the boundary.  Every call raises
RuntimeError with the library's status string when it returns a non-zero
status, mirroring the RuntimeError the reference's ttnn ops raise.  The product
path has no fallback: if the library cannot be loaded, the first call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libbitnet_b200.so")

BITNET_OK = 0
EPI_NONE, EPI_RELU2_MUL, EPI_RESIDUAL_ADD = 0, 1, 2
PATH_AUTO, PATH_SIMT, PATH_TCGEN05 = 0, 1, 2
MAX_SEGMENTS = 4

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_size_t = ctypes.c_size_t


class Segments(ctypes.Structure):
    """bitnet_segments_t: per-tensor scales of a fused projection."""

    _fields_ = [
        ("count", ctypes.c_int32),
        ("end", ctypes.c_int32 * MAX_SEGMENTS),
        ("scale", ctypes.c_float * MAX_SEGMENTS),
    ]

    @classmethod
    def make(cls, ends: list[int], scales: list[float]) -> "Segments":
        if not 1 <= len(scales) <= MAX_SEGMENTS or len(ends) != len(scales):
            raise ValueError("segments: 1..4 (end, scale) pairs expected")
        s = cls()
        s.count = len(scales)
        for i, (e, sc) in enumerate(zip(ends, scales)):
            s.end[i] = int(e)
            s.scale[i] = float(sc)
        return s


class DecodeLayer(ctypes.Structure):
    """bitnet_decode_layer_t."""

    _fields_ = [
        ("w_qkv", ctypes.c_void_p),
        ("w_o", ctypes.c_void_p),
        ("w_gate_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("seg_qkv", Segments),
        ("seg_o", Segments),
        ("seg_gate_up", Segments),
        ("seg_down", Segments),
        ("input_layernorm", ctypes.c_void_p),
        ("attn_sub_norm", ctypes.c_void_p),
        ("post_attention_layernorm", ctypes.c_void_p),
        ("ffn_sub_norm", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
    ]


class DecodeDesc(ctypes.Structure):
    """bitnet_decode_desc_t."""

    _fields_ = [
        ("num_layers", ctypes.c_int),
        ("batch", ctypes.c_int),
        ("hidden", ctypes.c_int),
        ("intermediate", ctypes.c_int),
        ("n_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("layers", ctypes.POINTER(DecodeLayer)),
        ("hidden_state", ctypes.c_void_p),
        ("qkv", ctypes.c_void_p),
        ("attn", ctypes.c_void_p),
        ("mid", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("rope_len", ctypes.c_int),
        ("max_len", ctypes.c_int),
        ("max_ctx", ctypes.c_int),
        ("attn_workspace", ctypes.c_void_p),
        ("attn_workspace_bytes", ctypes.c_size_t),
        ("splits", ctypes.c_int * 4),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "bitnet_abi_version": (_c_int, []),
    "bitnet_status_string": (ctypes.c_char_p, [_c_int]),
    "bitnet_last_device_status": (_c_int, [ctypes.POINTER(_c_int)]),
    "bitnet_last_cuda_error": (ctypes.c_char_p, []),
    "bitnet_set_pdl": (_c_int, [_c_int]),
    "bitnet_set_tc_split": (_c_int, [_c_int]),
    "bitnet_set_simt_max_m": (_c_int, [_c_int]),
    "bitnet_packed_weight_bytes": (_c_size_t, [_c_int, _c_int]),
    "bitnet_act_bytes": (_c_size_t, [_c_int, _c_int]),
    "bitnet_act_rows": (_c_int, [_c_int]),
    "bitnet_pack_ternary": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "bitnet_pack_from_canonical": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "bitnet_tilized_weight_bytes": (_c_size_t, [_c_int, _c_int]),
    "bitnet_pack_from_tilized": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "bitnet_act_quant": (
        _c_int,
        [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_float, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p],
    ),
    "bitnet_bitlinear_q": (
        _c_int,
        [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_int, ctypes.POINTER(Segments), _c_int,
         _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p],
    ),
    "bitnet_bitlinear": (
        _c_int,
        [_c_void_p, _c_int, _c_int, _c_void_p, _c_float, _c_void_p, _c_int, ctypes.POINTER(Segments), _c_int,
         _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p],
    ),
    "bitnet_bitlinear_noalloc": (
        _c_int,
        [_c_void_p, _c_int, _c_int, _c_void_p, _c_float, _c_void_p, _c_int, ctypes.POINTER(Segments), _c_int,
         _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p],
    ),
    "bitnet_gqa_decode_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "bitnet_gqa_decode_attention": (
        _c_int,
        [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p,
         _c_int, _c_int, _c_float, _c_void_p, _c_size_t, _c_void_p, _c_void_p],
    ),
    "bitnet_decode_plan_create": (_c_int, [ctypes.POINTER(DecodeDesc), ctypes.POINTER(_c_void_p)]),
    "bitnet_decode_plan_run": (_c_int, [_c_void_p, _c_void_p]),
    "bitnet_decode_plan_destroy": (_c_int, [_c_void_p]),
    "bitnet_lm_head_argmax_shard": (
        _c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p]),
    "bitnet_argmax_merge_pairs": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p]),
    "bitnet_rope_append_prefill": (
        _c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p,
                 _c_void_p, _c_int, _c_void_p]),
    "bitnet_attention_prefill": (
        _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_void_p,
                 _c_void_p]),
    "bitnet_rope_append_prefill_varlen": (
        _c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_int,
                 _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "bitnet_attention_prefill_varlen": (
        _c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float,
                 _c_void_p, _c_void_p]),
    "bitnet_selftest_bounded_wait": (_c_int, [ctypes.c_longlong, _c_void_p]),
    "bitnet_lm_head_bytes": (_c_size_t, [_c_int, _c_int]),
    "bitnet_pack_lm_head": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "bitnet_embed_gather": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "bitnet_argmax_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int]),
    "bitnet_lm_head_argmax": (
        _c_int,
        [_c_void_p, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    ),
}

_lib = None
_lock = threading.Lock()


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            p = path or LIB_PATH
            if not os.path.exists(p):
                raise RuntimeError(
                    f"{p} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                    "(the B200 path has no CPU fallback)"
                )
            lib = ctypes.CDLL(p)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def status_string(status: int) -> str:
    return load().bitnet_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != BITNET_OK:
        detail = ""
        if status == -4:
            detail = f" [{load().bitnet_last_cuda_error().decode()}]"
        raise RuntimeError(f"{what} failed: {status_string(status)} (status {status}){detail}")


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("bitnet-tt B200 kernels take CUDA tensors only (no CPU path)")
    return t.data_ptr()


def stream_handle(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def last_device_status() -> tuple[int, int]:
    site = _c_int(0)
    st = load().bitnet_last_device_status(ctypes.byref(site))
    return st, site.value


# ---------------------------------------------------------------------------
# thin typed wrappers
# ---------------------------------------------------------------------------
def packed_weight_bytes(n: int, k: int) -> int:
    return int(load().bitnet_packed_weight_bytes(n, k))


def act_bytes(m: int, k: int) -> int:
    return int(load().bitnet_act_bytes(m, k))


def act_rows(m: int) -> int:
    return int(load().bitnet_act_rows(m))


def set_pdl(enable: bool) -> None:
    check(load().bitnet_set_pdl(1 if enable else 0), "bitnet_set_pdl")


def set_tc_split(split: int) -> None:
    check(load().bitnet_set_tc_split(int(split)), "bitnet_set_tc_split")


def set_simt_max_m(m: int) -> None:
    check(load().bitnet_set_simt_max_m(int(m)), "bitnet_set_simt_max_m")


def pack_ternary(w_q: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """int8 ternary [N, K] (CUDA) -> device weight layout (uint8)."""
    if w_q.dtype != torch.int8 or w_q.dim() != 2:
        raise ValueError("pack_ternary expects an int8 [N, K] tensor")
    w_q = w_q.contiguous()
    n, k = w_q.shape
    if out is None:
        out = torch.empty(packed_weight_bytes(n, k), dtype=torch.uint8, device=w_q.device)
    check(load().bitnet_pack_ternary(ptr(w_q), n, k, ptr(out), stream_handle()), "bitnet_pack_ternary")
    return out


def pack_from_canonical(canonical: torch.Tensor, n: int, k: int) -> torch.Tensor:
    out = torch.empty(packed_weight_bytes(n, k), dtype=torch.uint8, device=canonical.device)
    check(load().bitnet_pack_from_canonical(ptr(canonical.contiguous()), n, k, ptr(out), stream_handle()),
          "bitnet_pack_from_canonical")
    return out


def tilized_weight_bytes(n: int, k: int) -> int:
    return int(load().bitnet_tilized_weight_bytes(n, k))


def pack_from_tilized(tiles: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """The reference's Tensix tile format (uint8 [tiles, 256], kernels/pack.py
    pack_ternary_tilized of W [n, k]) -> device weight layout."""
    if tiles.dtype != torch.uint8 or tiles.numel() != tilized_weight_bytes(n, k):
        raise ValueError("pack_from_tilized expects uint8 tiles of tilized_weight_bytes(n, k) bytes")
    out = torch.empty(packed_weight_bytes(n, k), dtype=torch.uint8, device=tiles.device)
    check(load().bitnet_pack_from_tilized(ptr(tiles.contiguous()), n, k, ptr(out), stream_handle()),
          "bitnet_pack_from_tilized")
    return out


class ActBuffers:
    """Caller-owned quantised-activation buffers for up to `m` tokens x `k` features."""

    def __init__(self, m: int, k: int, device: torch.device | str):
        self.m, self.k = m, k
        self.q = torch.empty(act_bytes(m, k), dtype=torch.int8, device=device)
        rows = act_rows(m)
        self.row_scale = torch.empty(rows, dtype=torch.float32, device=device)
        self.row_sum = torch.empty(rows, dtype=torch.int32, device=device)


def act_quant(x: torch.Tensor, gamma: torch.Tensor | None, eps: float, bufs: ActBuffers,
              normed_out: torch.Tensor | None = None) -> None:
    m, k = x.shape
    if x.dtype != torch.bfloat16:
        raise ValueError("activations must be bf16")
    check(load().bitnet_act_quant(ptr(x), m, k, x.stride(0), ptr(gamma), float(eps), ptr(bufs.q),
                                  ptr(bufs.row_scale), ptr(bufs.row_sum), ptr(normed_out), stream_handle()),
          "bitnet_act_quant")


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    m, k = x.shape
    if out is None:
        out = torch.empty((m, k), dtype=torch.bfloat16, device=x.device)
    check(load().bitnet_act_quant(ptr(x), m, k, x.stride(0), ptr(gamma), float(eps), None, None, None, ptr(out),
                                  stream_handle()), "bitnet_act_quant(rmsnorm)")
    return out


def bitlinear_q(bufs: ActBuffers, m: int, k: int, w_packed: torch.Tensor, n: int, segments: Segments | None,
                epilogue: int, residual: torch.Tensor | None, y: torch.Tensor, acc_out: torch.Tensor | None = None,
                path: int = PATH_AUTO) -> None:
    seg = ctypes.byref(segments) if segments is not None else None
    check(load().bitnet_bitlinear_q(ptr(bufs.q), ptr(bufs.row_scale), ptr(bufs.row_sum), m, k, ptr(w_packed), n,
                                    seg, epilogue, ptr(residual), ptr(y), ptr(acc_out), path, stream_handle()),
          "bitnet_bitlinear_q")


SIMT_FUSED_MAX_M = 4  # bitnet_bitlinear runs as one fused launch for M <= this (the CUDA-core path)


def bitlinear_fused(x: torch.Tensor, gamma: torch.Tensor | None, eps: float, bufs: ActBuffers, w_packed: torch.Tensor,
                    n: int, segments: Segments | None, epilogue: int, residual: torch.Tensor | None, y: torch.Tensor,
                    acc_out: torch.Tensor | None = None, path: int = PATH_AUTO) -> None:
    """bitnet_bitlinear: RMSNorm + act-quant + ternary contraction + epilogue.  For
    M <= SIMT_FUSED_MAX_M one kernel; otherwise the act-quant and BitLinear
    launches (bufs holds the codes)."""
    m, k = x.shape
    if x.dtype != torch.bfloat16 or x.stride(0) != k:
        raise ValueError("x must be contiguous bf16 [M, K]")
    seg = ctypes.byref(segments) if segments is not None else None
    check(load().bitnet_bitlinear(ptr(x), m, k, ptr(gamma), float(eps), ptr(w_packed), n, seg, epilogue,
                                  ptr(residual), ptr(y), ptr(acc_out), ptr(bufs.q), ptr(bufs.row_scale),
                                  ptr(bufs.row_sum), path, stream_handle()), "bitnet_bitlinear")


def gqa_decode_workspace_bytes(b: int, n_heads: int, n_kv: int, max_ctx: int) -> int:
    return int(load().bitnet_gqa_decode_workspace_bytes(b, n_heads, n_kv, max_ctx))


def gqa_decode_workspace(b: int, n_heads: int, n_kv: int, max_ctx: int, device) -> torch.Tensor | None:
    """Zeroed attention workspace (None when the context needs no split)."""
    nbytes = gqa_decode_workspace_bytes(b, n_heads, n_kv, max_ctx)
    return torch.zeros(nbytes, dtype=torch.uint8, device=device) if nbytes > 0 else None


def gqa_decode_attention(qkv: torch.Tensor, n_heads: int, n_kv: int, head_dim: int, positions: torch.Tensor,
                         rope_cos: torch.Tensor, rope_sin: torch.Tensor, k_cache: torch.Tensor,
                         v_cache: torch.Tensor, scale: float, out: torch.Tensor, max_ctx: int = 0,
                         workspace: torch.Tensor | None = None) -> None:
    b = qkv.shape[0]
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(load().bitnet_gqa_decode_attention(ptr(qkv), b, n_heads, n_kv, head_dim, ptr(positions), ptr(rope_cos),
                                             ptr(rope_sin), rope_cos.shape[0], ptr(k_cache), ptr(v_cache),
                                             k_cache.shape[2], int(max_ctx), float(scale), ptr(workspace), ws_bytes,
                                             ptr(out), stream_handle()),
          "bitnet_gqa_decode_attention")


def lm_head_bytes(v: int, k: int) -> int:
    return int(load().bitnet_lm_head_bytes(v, k))


def pack_lm_head(w: torch.Tensor) -> torch.Tensor:
    v, k = w.shape
    out = torch.empty(lm_head_bytes(v, k), dtype=torch.uint8, device=w.device)
    check(load().bitnet_pack_lm_head(ptr(w.contiguous()), v, k, ptr(out), stream_handle()), "bitnet_pack_lm_head")
    return out


def embed_gather(ids: torch.Tensor, w_tiled: torch.Tensor, v: int, k: int, out: torch.Tensor) -> None:
    check(load().bitnet_embed_gather(ptr(ids), ids.numel(), ptr(w_tiled), v, k, ptr(out), stream_handle()),
          "bitnet_embed_gather")


def argmax_workspace_bytes(b: int, k: int, v: int) -> int:
    return int(load().bitnet_argmax_workspace_bytes(b, k, v))


def lm_head_argmax(h: torch.Tensor, w_tiled: torch.Tensor, v: int, workspace: torch.Tensor, out_ids: torch.Tensor,
                   logits_out: torch.Tensor | None = None, advance_positions: torch.Tensor | None = None) -> None:
    b, k = h.shape
    check(load().bitnet_lm_head_argmax(ptr(h), b, k, ptr(w_tiled), v, ptr(workspace), ptr(out_ids),
                                       ptr(logits_out), ptr(advance_positions), stream_handle()),
          "bitnet_lm_head_argmax")


class DecodePlan:
    """All transformer layers of a decode step in one persistent launch
    (bitnet_decode_plan_*).  Holds references to every tensor it points at."""

    def __init__(self, model, hidden: torch.Tensor, qkv: torch.Tensor, attn: torch.Tensor, mid: torch.Tensor,
                 positions: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor, caches,
                 max_ctx: int = 0, attn_workspace: torch.Tensor | None = None,
                 splits: tuple[int, int, int, int] | None = None) -> None:
        cfg = model.config
        n = cfg.num_layers
        layers = (DecodeLayer * n)()
        keep = [hidden, qkv, attn, mid, positions, rope_cos, rope_sin, attn_workspace]
        for i, (blk, cache) in enumerate(zip(model.layers, caches)):
            at, mlp = blk.self_attn, blk.mlp
            L = layers[i]
            L.w_qkv, L.w_o = ptr(at.qkv_proj.weight), ptr(at.o_proj.weight)
            L.w_gate_up, L.w_down = ptr(mlp.gate_up_proj.weight), ptr(mlp.down_proj.weight)
            L.seg_qkv, L.seg_o = at.qkv_proj.segments(), at.o_proj.segments()
            L.seg_gate_up, L.seg_down = mlp.gate_up_proj.segments(), mlp.down_proj.segments()
            L.input_layernorm = ptr(blk.input_layernorm.weight)
            L.attn_sub_norm = ptr(at.attn_sub_norm.weight)
            L.post_attention_layernorm = ptr(blk.post_attention_layernorm.weight)
            L.ffn_sub_norm = ptr(mlp.ffn_sub_norm.weight)
            L.k_cache, L.v_cache = ptr(cache.key_cache), ptr(cache.value_cache)
            keep += [at.qkv_proj.weight, at.o_proj.weight, mlp.gate_up_proj.weight, mlp.down_proj.weight,
                     cache.key_cache, cache.value_cache]
        d = DecodeDesc()
        d.num_layers, d.batch, d.hidden = n, hidden.shape[0], cfg.hidden_size
        d.intermediate, d.n_heads, d.n_kv_heads = cfg.intermediate_size, cfg.num_attention_heads, cfg.num_key_value_heads
        d.head_dim, d.eps = cfg.head_dim, cfg.rms_norm_eps
        d.layers = layers
        d.hidden_state, d.qkv, d.attn, d.mid = ptr(hidden), ptr(qkv), ptr(attn), ptr(mid)
        d.positions, d.rope_cos, d.rope_sin = ptr(positions), ptr(rope_cos), ptr(rope_sin)
        d.rope_len, d.max_len, d.max_ctx = rope_cos.shape[0], caches[0].key_cache.shape[2], int(max_ctx)
        d.attn_workspace = ptr(attn_workspace)
        d.attn_workspace_bytes = attn_workspace.numel() if attn_workspace is not None else 0
        for i, v in enumerate(splits or (0, 0, 0, 0)):
            d.splits[i] = int(v)
        h = _c_void_p()
        check(load().bitnet_decode_plan_create(ctypes.byref(d), ctypes.byref(h)), "bitnet_decode_plan_create")
        self._h = h
        self._keep = keep

    def run(self) -> None:
        check(load().bitnet_decode_plan_run(self._h, stream_handle()), "bitnet_decode_plan_run")

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            load().bitnet_decode_plan_destroy(self._h)
            self._h = _c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def lm_head_argmax_shard(h: torch.Tensor, w_tiled_shard: torch.Tensor, v_shard: int, vocab_offset: int,
                         workspace: torch.Tensor, pairs_out: torch.Tensor) -> None:
    """pairs_out: float32 [B, 2] viewed as {value, int32 index} (see the C header)."""
    b, k = h.shape
    check(load().bitnet_lm_head_argmax_shard(ptr(h), b, k, ptr(w_tiled_shard), v_shard, vocab_offset, ptr(workspace),
                                             ptr(pairs_out), stream_handle()), "bitnet_lm_head_argmax_shard")


def argmax_merge_pairs(pairs: torch.Tensor, out_ids: torch.Tensor, advance_positions: torch.Tensor | None = None) -> None:
    """pairs: [nshard, B, 2] float32 pairs as written by lm_head_argmax_shard."""
    nshard, b = pairs.shape[0], pairs.shape[1]
    check(load().bitnet_argmax_merge_pairs(ptr(pairs), nshard, b, ptr(out_ids), ptr(advance_positions),
                                           stream_handle()), "bitnet_argmax_merge_pairs")


def rope_append_prefill(qkv: torch.Tensor, b: int, p: int, n_heads: int, n_kv: int, rope_cos: torch.Tensor,
                        rope_sin: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    check(load().bitnet_rope_append_prefill(ptr(qkv), b, p, n_heads, n_kv, 128, ptr(rope_cos), ptr(rope_sin),
                                            rope_cos.shape[0], ptr(q_out), ptr(k_cache), ptr(v_cache),
                                            k_cache.shape[2], stream_handle()), "bitnet_rope_append_prefill")


def attention_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, b: int, p: int, n_heads: int,
                      n_kv: int, scale: float, out: torch.Tensor) -> None:
    check(load().bitnet_attention_prefill(ptr(q), ptr(k_cache), ptr(v_cache), b, p, n_heads, n_kv, 128,
                                          k_cache.shape[2], float(scale), ptr(out), stream_handle()),
          "bitnet_attention_prefill")


def rope_append_prefill_varlen(qkv: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int, n_heads: int, n_kv: int,
                               rope_cos: torch.Tensor, rope_sin: torch.Tensor, q_out: torch.Tensor,
                               k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    b = cu_seqlens.numel() - 1
    check(load().bitnet_rope_append_prefill_varlen(ptr(qkv), b, ptr(cu_seqlens), qkv.shape[0], int(max_seqlen), n_heads,
                                                   n_kv, 128, ptr(rope_cos), ptr(rope_sin), rope_cos.shape[0],
                                                   ptr(q_out), ptr(k_cache), ptr(v_cache), k_cache.shape[2],
                                                   stream_handle()), "bitnet_rope_append_prefill_varlen")


def attention_prefill_varlen(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cu_seqlens: torch.Tensor,
                             max_seqlen: int, n_heads: int, n_kv: int, scale: float, out: torch.Tensor) -> None:
    b = cu_seqlens.numel() - 1
    check(load().bitnet_attention_prefill_varlen(ptr(q), ptr(k_cache), ptr(v_cache), b, ptr(cu_seqlens),
                                                 int(max_seqlen), n_heads, n_kv, 128, k_cache.shape[2], float(scale),
                                                 ptr(out), stream_handle()), "bitnet_attention_prefill_varlen")
