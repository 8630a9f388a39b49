"""Weight loading (mirrors src/bitnet_tt/utils/weights.py of the reference) and
the seeded synthetic BitNet-2B-shaped state dicts used by the benches.

load_bitnet_weights reads a local HF checkpoint directory (config.json +
*.safetensors); converting keys, splitting per layer and loading into a model
follow the reference functions of the same names.  No checkpoint ships with
this build, so the benches and tests use synthetic_state_dict: a lazy mapping
that generates each tensor from (seed, key) on first access.
"""

from __future__ import annotations

import json
import os
import zlib
from collections.abc import Mapping
from typing import Any, Iterator

import numpy as np
import torch

from ..config import BitNet2B4TConfig, BitNetConfig

_TOP_LEVEL = {"model.embed_tokens.weight": "embed_tokens.weight", "model.norm.weight": "norm.weight",
              "lm_head.weight": "lm_head.weight"}


def load_bitnet_weights(model_id: str = "microsoft/bitnet-b1.58-2B-4T-bf16", cache_dir: str | None = None):
    """(state dict of numpy arrays with converted keys, config) from a checkpoint.

    `model_id` is a local directory, or a hub id already present in the local
    HF cache (there is no network access on the build or GPU hosts)."""
    path = model_id
    if not os.path.isdir(path):
        try:
            from huggingface_hub import snapshot_download

            path = snapshot_download(model_id, cache_dir=cache_dir, local_files_only=True,
                                     allow_patterns=["*.safetensors", "config.json"])
        except Exception as e:  # pragma: no cover - depends on the local cache
            raise FileNotFoundError(f"checkpoint {model_id!r} not found locally: {e}") from e
    with open(os.path.join(path, "config.json")) as f:
        hf = json.load(f)
    config = BitNet2B4TConfig(
        hidden_size=hf.get("hidden_size", 2560), num_layers=hf.get("num_hidden_layers", 30),
        num_attention_heads=hf.get("num_attention_heads", 20), num_key_value_heads=hf.get("num_key_value_heads", 5),
        intermediate_size=hf.get("intermediate_size", 6912), vocab_size=hf.get("vocab_size", 128256),
        max_position_embeddings=hf.get("max_position_embeddings", 4096), rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
        rope_theta=hf.get("rope_theta", 500000.0))
    from safetensors import safe_open

    raw: dict[str, np.ndarray] = {}
    for name in sorted(os.listdir(path)):
        if name.endswith(".safetensors"):
            with safe_open(os.path.join(path, name), framework="pt") as f:
                for key in f.keys():
                    raw[key] = f.get_tensor(key).float().numpy()
    return convert_hf_state_dict(raw), config


def convert_hf_state_dict(hf_state_dict: Mapping[str, Any]) -> dict[str, Any]:
    """HF keys -> the reference's keys: the embedding, final norm and layer keys
    drop their "model." prefix; every other key is kept unchanged."""
    out: dict[str, Any] = {}
    for key, value in hf_state_dict.items():
        if key in _TOP_LEVEL:
            out[_TOP_LEVEL[key]] = value
        elif key.startswith("model.layers."):
            out[key[len("model."):]] = value
        else:
            out[key] = value
    return out


def get_layer_weights(state_dict: Mapping[str, Any], layer_idx: int) -> dict[str, Any]:
    prefix = f"layers.{layer_idx}."
    return {k[len(prefix):]: state_dict[k] for k in state_dict.keys() if k.startswith(prefix)}


def save_numpy_weights(state_dict: Mapping[str, np.ndarray], output_path: str) -> None:
    np.savez_compressed(output_path, **{k: np.asarray(v) for k, v in state_dict.items()})


def load_numpy_weights(input_path: str) -> dict[str, np.ndarray]:
    data = np.load(input_path)
    return {k: data[k] for k in data.files}


def load_weights_to_model(model: Any, state_dict: Mapping[str, Any]) -> None:
    """Embedding, every layer, then the final norm and the lm_head (tied to the
    embedding when the state dict has no lm_head.weight)."""
    if "embed_tokens.weight" in state_dict:
        model.load_embedding_weights(state_dict["embed_tokens.weight"])
    for i in range(len(model.layers)):
        lw = get_layer_weights(state_dict, i)
        if lw:
            model.load_layer_weights(i, lw)
    if "norm.weight" in state_dict:
        lm = state_dict["lm_head.weight"] if "lm_head.weight" in state_dict else None
        model.load_final_weights(state_dict["norm.weight"], lm)


# ---------------------------------------------------------------------------
# synthetic weights (random init of the 2B-4T shape)
# ---------------------------------------------------------------------------
def layer_shapes(config: BitNetConfig) -> dict[str, tuple[int, ...]]:
    h, f, d = config.hidden_size, config.intermediate_size, config.head_dim
    nq, nkv = config.num_attention_heads * d, config.num_key_value_heads * d
    return {
        "input_layernorm.weight": (h,), "post_attention_layernorm.weight": (h,),
        "self_attn.q_proj.weight": (nq, h), "self_attn.k_proj.weight": (nkv, h),
        "self_attn.v_proj.weight": (nkv, h), "self_attn.o_proj.weight": (h, nq),
        "self_attn.attn_sub_norm.weight": (h,), "mlp.gate_proj.weight": (f, h), "mlp.up_proj.weight": (f, h),
        "mlp.down_proj.weight": (h, f), "mlp.ffn_sub_norm.weight": (f,),
    }


class SyntheticStateDict(Mapping):
    """Lazy, seeded BitNet state dict (reference key names, converted form).

    Linear weights are latent W ~ N(0, linear_std) float32 (quantised at load
    time to ternary with scale mean|W|); embeddings ~ N(0, embed_std) and norm
    weights 1 + norm_noise * N(0, 1) are rounded to bf16.  Each tensor is a
    deterministic function of (seed, key), generated on `device` when read.
    """

    def __init__(self, config: BitNetConfig, seed: int = 0, device: str | torch.device = "cpu",
                 linear_std: float = 0.02, embed_std: float = 0.02, norm_noise: float = 0.1):
        self.config, self.seed, self.device = config, seed, torch.device(device)
        self.linear_std, self.embed_std, self.norm_noise = linear_std, embed_std, norm_noise
        self._shapes: dict[str, tuple[int, ...]] = {
            "embed_tokens.weight": (config.vocab_size, config.hidden_size), "norm.weight": (config.hidden_size,)}
        for i in range(config.num_layers):
            for k, s in layer_shapes(config).items():
                self._shapes[f"layers.{i}.{k}"] = s

    def __len__(self) -> int:
        return len(self._shapes)

    def __iter__(self) -> Iterator[str]:
        return iter(self._shapes)

    def shape(self, key: str) -> tuple[int, ...]:
        return self._shapes[key]

    def __getitem__(self, key: str) -> torch.Tensor:
        shape = self._shapes[key]
        g = torch.Generator(device=self.device)
        g.manual_seed((self.seed * 1_000_003 + zlib.crc32(key.encode())) & 0x7FFFFFFFFFFF)
        x = torch.randn(shape, generator=g, device=self.device, dtype=torch.float32)
        if key.endswith("norm.weight") or key.endswith("layernorm.weight"):
            return (1.0 + self.norm_noise * x).to(torch.bfloat16).float()
        if key == "embed_tokens.weight":
            return (self.embed_std * x).to(torch.bfloat16).float()
        return self.linear_std * x


def synthetic_state_dict(config: BitNetConfig, seed: int = 0, device: str | torch.device = "cpu",
                         **kw) -> SyntheticStateDict:
    return SyntheticStateDict(config, seed, device, **kw)
