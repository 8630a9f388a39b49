"""Rotary position tables.

precompute_freqs_cis keeps the reference's NumPy helper
(src/bitnet_tt/utils/rope.py:7-22, interleaved [f0, f0, f1, f1, ...] layout).
The decode kernel uses the HF half-split convention
(transformers BitNetRotaryEmbedding + apply_rotary_pos_emb): cos/sin of
pos * inv_freq computed in fp32 and cast to the model dtype (bf16); the table
stores the 64 distinct frequencies per position.
"""

from __future__ import annotations

import numpy as np
import torch


def precompute_freqs_cis(dim: int, max_seq_len: int, theta: float = 10000.0):
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    ang = np.repeat(np.arange(max_seq_len, dtype=np.float32)[:, None] * inv[None, :], 2, axis=-1)
    return (np.cos(ang).astype(np.float32).reshape(1, 1, max_seq_len, dim),
            np.sin(ang).astype(np.float32).reshape(1, 1, max_seq_len, dim))


def half_split_tables(head_dim: int, max_len: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos/sin tables [max_len, head_dim // 2] for the HF half-split RoPE."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim
    inv_freq = 1.0 / (theta ** exps)
    ang = torch.arange(max_len, dtype=torch.float32)[:, None] * inv_freq[None, :]
    return ang.cos().to(torch.bfloat16).contiguous(), ang.sin().to(torch.bfloat16).contiguous()
