"""GQA attention with fused QKV BitLinear, decode kernel and KV cache.

Mirrors the reference's src/bitnet_tt/layers/attention.py: KVCache (116-458),
build_fused_qkv_weight (481-506), MultiHeadAttention.load_weights (776-839) and
the decode path _forward_decode_1bkd (1040-1262).  On the B200 the decode step
is: fused-norm QKV BitLinear (three per-projection scales applied in the
epilogue) -> one attention kernel (half-split RoPE on Q and K, K/V append at
the sequence's position, GQA softmax attention) -> attn_sub_norm fused into
the o_proj BitLinear, whose epilogue adds the residual.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _lib
from .bitlinear import Linear, RMSNorm, quantize_and_transpose_weight, quantize_ternary


def _permute_halfsplit_to_adjacent(weight_t: np.ndarray, num_heads: int, head_dim: int) -> np.ndarray:
    """Reference attention.py:462-478: column order for the adjacent-pair RoPE of
    Tensix; the B200 kernel uses the half-split order and never needs it."""
    half = head_dim // 2
    perm = np.stack([np.arange(half), np.arange(half) + half], axis=1).reshape(-1)
    out = weight_t.copy()
    for h in range(num_heads):
        out[:, h * head_dim:(h + 1) * head_dim] = weight_t[:, h * head_dim + perm]
    return out


def build_fused_qkv_weight(q_weight, k_weight, v_weight, num_heads: int = 0, num_kv_heads: int = 0,
                           head_dim: int = 0, permute_for_rope: bool = False):
    """Pre-transposed ternary [in, q + k + v] and the three per-projection scales
    (reference attention.py:481-506)."""
    q_t, q_s = quantize_and_transpose_weight(np.asarray(q_weight))
    k_t, k_s = quantize_and_transpose_weight(np.asarray(k_weight))
    v_t, v_s = quantize_and_transpose_weight(np.asarray(v_weight))
    if permute_for_rope and head_dim > 0:
        q_t = _permute_halfsplit_to_adjacent(q_t, num_heads, head_dim)
        k_t = _permute_halfsplit_to_adjacent(k_t, num_kv_heads, head_dim)
    return np.concatenate([q_t, k_t, v_t], axis=1), q_s, k_s, v_s


class KVCache:
    """bf16 K/V cache [batch, n_kv_heads, max_seq_len, head_dim] for one layer."""

    def __init__(self, max_seq_len: int, batch_size: int, num_kv_heads: int, head_dim: int, device=None):
        self.max_seq_len = max_seq_len
        self.batch_size = batch_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.device = torch.device(device if device is not None else "cuda")
        self.key_cache: torch.Tensor | None = None
        self.value_cache: torch.Tensor | None = None
        self.seq_len_cached = 0

    def preallocate(self, **_ignored) -> None:
        shape = (self.batch_size, self.num_kv_heads, self.max_seq_len, self.head_dim)
        self.key_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.value_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)

    def reset(self) -> None:
        self.seq_len_cached = 0

    def attention_workspace(self, num_heads: int, max_ctx: int = 0) -> torch.Tensor | None:
        """Zeroed split-context workspace of the decode attention kernel (None
        when max_ctx needs no split); cached per size, the kernel leaves it zeroed."""
        max_ctx = max_ctx or self.max_seq_len
        nbytes = _lib.gqa_decode_workspace_bytes(self.batch_size, num_heads, self.num_kv_heads, max_ctx)
        if nbytes == 0:
            return None
        ws = getattr(self, "_attn_ws", None)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._attn_ws = ws
        return ws

    def clear(self) -> None:
        self.key_cache = None
        self.value_cache = None
        self.seq_len_cached = 0


class MultiHeadAttention:
    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, device=None, eps: float = 1e-5,
                 max_seq_len: int = 4096, rope_theta: float = 500000.0, weight_dtype: str = "packed_ternary",
                 use_fused_rope: bool = True, **_ignored) -> None:
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = hidden_size // num_heads
        self.device = torch.device(device if device is not None else "cuda")
        self.scale = self.head_dim ** -0.5
        self.use_fused_rope = use_fused_rope
        self._qkv_dim = (num_heads + 2 * num_kv_heads) * self.head_dim
        self.qkv_proj = Linear(hidden_size, self._qkv_dim, self.device, weight_dtype=weight_dtype)
        self.o_proj = Linear(num_heads * self.head_dim, hidden_size, self.device, weight_dtype=weight_dtype)
        self.attn_sub_norm = RMSNorm(hidden_size, self.device, eps)
        self._qkv_scales = (1.0, 1.0, 1.0)
        self._qkv_use_packed_ternary = True

    @property
    def qkv_fused_weight(self) -> torch.Tensor | None:
        return self.qkv_proj.weight

    def load_weights(self, q_weight, k_weight, v_weight, o_weight, attn_sub_norm_weight=None) -> None:
        qq, qs = quantize_ternary(q_weight)
        kq, ks = quantize_ternary(k_weight)
        vq, vs = quantize_ternary(v_weight)
        nq, nk = qq.shape[0], kq.shape[0]
        fused = torch.cat([qq.to(self.device), kq.to(self.device), vq.to(self.device)], dim=0)
        self.qkv_proj.load_ternary(fused, 1.0, segments=[(nq, qs), (nq + nk, ks), (self._qkv_dim, vs)])
        self._qkv_scales = (qs, ks, vs)
        self.o_proj.load_weights(o_weight)
        if attn_sub_norm_weight is not None:
            self.attn_sub_norm.load_weights(attn_sub_norm_weight)

    def decode_attention(self, qkv: torch.Tensor, positions: torch.Tensor, rope_cos: torch.Tensor,
                         rope_sin: torch.Tensor, cache: KVCache, out: torch.Tensor, max_ctx: int = 0,
                         workspace: torch.Tensor | None = None) -> None:
        """RoPE + KV append + GQA attention for one token per sequence.  max_ctx
        bounds positions + 1 (0: the cache length) and sets the context split."""
        if workspace is None:
            workspace = cache.attention_workspace(self.num_heads, max_ctx)
        _lib.gqa_decode_attention(qkv, self.num_heads, self.num_kv_heads, self.head_dim, positions, rope_cos,
                                  rope_sin, cache.key_cache, cache.value_cache, self.scale, out, max_ctx, workspace)

    def __call__(self, hidden_states: torch.Tensor, positions: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor],
                 cache: KVCache, norm_weight: torch.Tensor | None = None, norm_epsilon: float = 1e-5,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
        """Decode forward for [batch, hidden] (one new token per sequence)."""
        qkv = self.qkv_proj(hidden_states, norm_weight=norm_weight, norm_epsilon=norm_epsilon)
        attn = torch.empty((qkv.shape[0], self.num_heads * self.head_dim), dtype=torch.bfloat16, device=qkv.device)
        self.decode_attention(qkv, positions, rope[0], rope[1], cache, attn)
        return self.o_proj(attn, norm_weight=self.attn_sub_norm.weight, norm_epsilon=self.attn_sub_norm.eps,
                           residual=residual)
