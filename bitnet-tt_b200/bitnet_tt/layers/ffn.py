"""Gated FFN: fused gate/up BitLinear with the ReLU^2(gate) * up epilogue, then
ffn_sub_norm fused into the down BitLinear.

Mirrors the reference's src/bitnet_tt/layers/ffn.py (build_fused_gate_up_weight
22-34, FeedForward 37-183).  On the B200 the fused gate/up matrix stores its
rows in 64-row groups [32 gate rows | the matching 32 up rows], so one CTA of
the BitLinear owns both halves of every output and applies
h = bf16(bf16(relu(g)^2) * u) before anything leaves the chip; gate and up keep
their own per-tensor scales (HF AutoBitLinear semantics).
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _lib
from .bitlinear import Linear, RMSNorm, quantize_and_transpose_weight, quantize_ternary


def build_fused_gate_up_weight(gate_weight, up_weight):
    """Pre-transposed ternary [in, 2F] = gate^T | up^T and the two scales
    (reference ffn.py:22-34)."""
    g_t, g_s = quantize_and_transpose_weight(np.asarray(gate_weight))
    u_t, u_s = quantize_and_transpose_weight(np.asarray(up_weight))
    return np.concatenate([g_t, u_t], axis=1), g_s, u_s


def interleave_gate_up(gate_q: torch.Tensor, up_q: torch.Tensor) -> torch.Tensor:
    """[F, H] gate and up codes -> [2F, H] in 64-row groups [32 gate | 32 up]."""
    f, h = gate_q.shape
    if f % 32:
        raise ValueError("intermediate size must be a multiple of 32")
    return torch.stack([gate_q.reshape(f // 32, 32, h), up_q.reshape(f // 32, 32, h)], dim=1).reshape(2 * f, h)


class FeedForward:
    def __init__(self, hidden_size: int, intermediate_size: int, device=None, eps: float = 1e-5,
                 model_config=None, use_lofi: bool = False, weight_dtype: str = "packed_ternary") -> None:
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.device = torch.device(device if device is not None else "cuda")
        self.eps = eps
        self.gate_up_proj = Linear(hidden_size, 2 * intermediate_size, self.device, weight_dtype=weight_dtype)
        self.gate_up_proj.epilogue = _lib.EPI_RELU2_MUL
        self.down_proj = Linear(intermediate_size, hidden_size, self.device, weight_dtype=weight_dtype)
        self.ffn_sub_norm = RMSNorm(intermediate_size, self.device, eps)
        self._gate_scale = 1.0
        self._up_scale = 1.0

    def load_weights(self, gate_weight, up_weight, down_weight, ffn_sub_norm_weight=None) -> None:
        gq, gs = quantize_ternary(gate_weight)
        uq, us = quantize_ternary(up_weight)
        fused = interleave_gate_up(gq.to(self.device), uq.to(self.device))
        self.gate_up_proj.load_ternary(fused, 1.0, segments=[(self.intermediate_size, gs),
                                                             (2 * self.intermediate_size, us)])
        self._gate_scale, self._up_scale = gs, us
        self.down_proj.load_weights(down_weight)
        if ffn_sub_norm_weight is not None:
            self.ffn_sub_norm.load_weights(ffn_sub_norm_weight)

    def __call__(self, x: torch.Tensor, mode: str = "decode", norm_weight: torch.Tensor | None = None,
                 norm_epsilon: float = 1e-5, residual: torch.Tensor | None = None) -> torch.Tensor:
        hidden = self.gate_up_proj(x, norm_weight=norm_weight, norm_epsilon=norm_epsilon)
        return self.down_proj(hidden, norm_weight=self.ffn_sub_norm.weight, norm_epsilon=self.ffn_sub_norm.eps,
                              residual=residual)
