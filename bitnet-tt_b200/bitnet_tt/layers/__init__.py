"""Layers: BitLinear, RMSNorm, attention, FFN, embedding."""

from .attention import KVCache, MultiHeadAttention, build_fused_qkv_weight  # noqa: F401
from .bitlinear import Linear, RMSNorm, quantize_and_transpose_weight  # noqa: F401
from .embedding import Embedding  # noqa: F401
from .ffn import FeedForward, build_fused_gate_up_weight  # noqa: F401
