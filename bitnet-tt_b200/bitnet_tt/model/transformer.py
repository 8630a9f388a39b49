"""Decoder block (mirrors src/bitnet_tt/model/transformer.py:59-254 of the reference).

Order (HF BitNetDecoderLayer): h += o_proj(attn_sub_norm(attn(input_layernorm(h))));
h += down(ffn_sub_norm(relu2(gate(n)) * up(n))) with n = post_attention_layernorm(h).
Every RMSNorm is fused into the BitLinear that consumes it, and both residual
adds are fused into the epilogues of o_proj and down.
"""

from __future__ import annotations

import torch

from ..config import BitNetConfig
from ..layers.attention import KVCache, MultiHeadAttention
from ..layers.bitlinear import RMSNorm
from ..layers.ffn import FeedForward


class TransformerBlock:
    def __init__(self, config: BitNetConfig, device=None, layer_idx: int = 0, weight_dtype: str = "packed_ternary",
                 use_fused_rope: bool = True, **_ignored) -> None:
        self.config = config
        self.layer_idx = layer_idx
        self.device = torch.device(device if device is not None else "cuda")
        eps = config.rms_norm_eps
        self.input_layernorm = RMSNorm(config.hidden_size, self.device, eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, self.device, eps)
        self.self_attn = MultiHeadAttention(config.hidden_size, config.num_attention_heads,
                                            config.num_key_value_heads, self.device, eps,
                                            config.max_position_embeddings, config.rope_theta, weight_dtype,
                                            use_fused_rope)
        self.mlp = FeedForward(config.hidden_size, config.intermediate_size, self.device, eps,
                               weight_dtype=weight_dtype)

    def load_weights(self, w: dict) -> None:
        self.input_layernorm.load_weights(w["input_layernorm.weight"])
        self.post_attention_layernorm.load_weights(w["post_attention_layernorm.weight"])
        self.self_attn.load_weights(w["self_attn.q_proj.weight"], w["self_attn.k_proj.weight"],
                                    w["self_attn.v_proj.weight"], w["self_attn.o_proj.weight"],
                                    w.get("self_attn.attn_sub_norm.weight"))
        self.mlp.load_weights(w["mlp.gate_proj.weight"], w["mlp.up_proj.weight"], w["mlp.down_proj.weight"],
                              w.get("mlp.ffn_sub_norm.weight"))

    def __call__(self, hidden: torch.Tensor, positions: torch.Tensor, rope, cache: KVCache) -> torch.Tensor:
        """Eager decode of one token per sequence; returns the new hidden state."""
        eps = self.config.rms_norm_eps
        h = self.self_attn(hidden, positions, rope, cache, norm_weight=self.input_layernorm.weight,
                           norm_epsilon=eps, residual=hidden)
        return self.mlp(h, norm_weight=self.post_attention_layernorm.weight, norm_epsilon=eps, residual=h)
