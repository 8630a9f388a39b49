"""Model configurations (mirrors src/bitnet_tt/config.py:13-46, 130-174 of the reference).

Only the architecture fields are kept; the Tenstorrent memory/compute-kernel
configs of the reference (get_model_config, get_compute_kernel_config) have no
B200 counterpart -- the CUDA kernels choose their own launch shapes.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class BitNetConfig:
    hidden_size: int = 2560
    num_layers: int = 30
    num_attention_heads: int = 20
    num_key_value_heads: int = 5
    intermediate_size: int = 6912
    vocab_size: int = 128256
    max_position_embeddings: int = 4096
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    weight_bits: int = 2
    activation_bits: int = 8
    hidden_act: str = "relu2"
    tie_word_embeddings: bool = True
    use_cache: bool = True
    attention_dropout: float = 0.0
    attention_bias: bool = False
    bos_token_id: int = 128000
    eos_token_id: int = 128001

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def num_kv_heads(self) -> int:
        return self.num_key_value_heads


@dataclass
class BitNetMiniConfig(BitNetConfig):
    """Small test model (reference config.py:130-144)."""

    hidden_size: int = 256
    num_layers: int = 4
    num_attention_heads: int = 4
    num_key_value_heads: int = 2
    intermediate_size: int = 512
    vocab_size: int = 1000
    max_position_embeddings: int = 512


@dataclass
class BitNet2B4TConfig(BitNetConfig):
    """microsoft/bitnet-b1.58-2B-4T shape (reference config.py:147-171)."""


def get_config(model_name: str = "mini") -> BitNetConfig:
    """reference config.py:174-197."""
    table = {"mini": BitNetMiniConfig, "2b4t": BitNet2B4TConfig, "2b": BitNet2B4TConfig, "base": BitNetConfig}
    key = model_name.lower()
    if key not in table:
        raise ValueError(f"Unknown model name: {model_name}. Choose from {sorted(table)}")
    return table[key]()
