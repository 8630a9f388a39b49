"""Load-time weight and activation quantisers with the reference's API
(src/bitnet_tt/utils/quantization.py of deveworld/bitnet-tt).

These run once at load time, on the host, exactly as in the reference.  The
per-token activation quantisation of the decode hot path runs on the GPU
(bitnet_act_quant in the C ABI); activation_quant_absmax here is the host form
the reference exposes for preprocessing and tests.
"""

from __future__ import annotations

import numpy as np
from numpy.typing import NDArray


def compute_weight_scale(weight: NDArray[np.floating], eps: float = 1e-5) -> np.floating:
    """Absmean scale gamma = max(mean(|W|), eps)."""
    return np.maximum(np.abs(weight).mean(), eps)


def weight_quant_ternary(weight: NDArray[np.floating], eps: float = 1e-5):
    """Ternary absmean quantisation: (clip(round(W / gamma), -1, 1) as int8, gamma)."""
    gamma = compute_weight_scale(weight, eps)
    return np.clip(np.round(weight / gamma), -1, 1).astype(np.int8), gamma


def activation_quant_absmax(x: NDArray[np.floating], num_bits: int = 8, eps: float = 1e-5):
    """Per-token absmax quantisation to [-2^(b-1), 2^(b-1) - 1]: (q int8, scale)."""
    top = 2 ** (num_bits - 1) - 1
    scale = top / np.maximum(np.abs(x).max(axis=-1, keepdims=True), eps)
    return np.clip(np.round(x * scale), -top - 1, top).astype(np.int8), scale


def dequantize_weight(weight_quant: NDArray[np.int8], scale: np.floating) -> NDArray[np.floating]:
    return weight_quant.astype(np.float32) * float(scale)


def pack_ternary_weights(weight_quant: NDArray[np.int8]) -> NDArray[np.uint8]:
    """Canonical 2-bit format: flattened codes (w + 1), four per byte, MSB first,
    padded with zero-weight codes."""
    codes = (weight_quant.astype(np.uint8).ravel() + np.uint8(1)) & np.uint8(3)
    codes = np.pad(codes, (0, (-codes.size) % 4), constant_values=1).reshape(-1, 4)
    weights = np.array([64, 16, 4, 1], dtype=np.uint8)
    return (codes * weights).sum(axis=1, dtype=np.uint16).astype(np.uint8)


def unpack_ternary_weights(packed: NDArray[np.uint8], original_shape: tuple[int, ...]) -> NDArray[np.int8]:
    shifts = np.array([6, 4, 2, 0], dtype=np.uint8)
    codes = (packed[:, None] >> shifts) & np.uint8(3)
    count = int(np.prod(original_shape))
    return (codes.ravel()[:count].astype(np.int8) - 1).reshape(original_shape)
