"""Weight loading (mirrors src/bitnet_tt/utils/weights.py of the reference) and
the seeded synthetic BitNet-2B-shaped state dicts used by the benches.

load_bitnet_weights reads a local HF checkpoint directory (config.json +
*.safetensors); converting keys, splitting per layer and loading into a model
follow the reference functions of the same names.  save_hf_checkpoint writes
such a directory; save_packed_weights / load_packed_weights cache a loaded
model in its device layout.  No checkpoint ships with this build, so the
benches and tests use synthetic_state_dict: a lazy mapping that generates each
tensor from (seed, key) on first access.
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
# checkpoints on disk: HF layout in, packed device layout cached
# ---------------------------------------------------------------------------
def save_hf_checkpoint(state_dict: Mapping[str, Any], config: BitNetConfig, path: str,
                       max_shard_bytes: int = 1 << 30) -> list[str]:
    """Write a state dict with this package's keys as an HF checkpoint directory:
    config.json plus bf16 ``model-XXXXX-of-YYYYY.safetensors`` shards with the HF
    key names (the inverse of load_bitnet_weights).  No real checkpoint ships
    with this build; tests and users write synthetic ones with it."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    inv = {v: k for k, v in _TOP_LEVEL.items()}
    tensors: list[tuple[str, torch.Tensor]] = []
    for key in state_dict.keys():
        hf_key = inv.get(key, "model." + key if key.startswith("layers.") else key)
        v = state_dict[key]
        t = v if isinstance(v, torch.Tensor) else torch.from_numpy(np.asarray(v, dtype=np.float32))
        tensors.append((hf_key, t.detach().to("cpu", torch.bfloat16).contiguous()))
    shards: list[list[tuple[str, torch.Tensor]]] = [[]]
    size = 0
    for name, t in tensors:
        nb = t.numel() * t.element_size()
        if shards[-1] and size + nb > max_shard_bytes:
            shards.append([])
            size = 0
        shards[-1].append((name, t))
        size += nb
    files = []
    for i, shard in enumerate(shards):
        fname = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(dict(shard), os.path.join(path, fname), metadata={"format": "pt"})
        files.append(fname)
    hf = {"architectures": ["BitNetForCausalLM"], "hidden_size": config.hidden_size,
          "num_hidden_layers": config.num_layers, "num_attention_heads": config.num_attention_heads,
          "num_key_value_heads": config.num_key_value_heads, "intermediate_size": config.intermediate_size,
          "vocab_size": config.vocab_size, "max_position_embeddings": config.max_position_embeddings,
          "rms_norm_eps": config.rms_norm_eps, "rope_theta": config.rope_theta, "torch_dtype": "bfloat16"}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
    return files


_PACKED_FORMAT = "bitnet-b200-packed-v1"


def _model_parts(model: Any) -> Iterator[tuple[str, str, Any]]:
    """(name, kind, object) of every device-resident weight of a model."""
    for i, layer in enumerate(model.layers):
        a, f = layer.self_attn, layer.mlp
        for name, lin in (("self_attn.qkv_proj", a.qkv_proj), ("self_attn.o_proj", a.o_proj),
                          ("mlp.gate_up_proj", f.gate_up_proj), ("mlp.down_proj", f.down_proj)):
            yield f"layers.{i}.{name}", "linear", lin
        for name, norm in (("input_layernorm", layer.input_layernorm),
                           ("post_attention_layernorm", layer.post_attention_layernorm),
                           ("self_attn.attn_sub_norm", a.attn_sub_norm), ("mlp.ffn_sub_norm", f.ffn_sub_norm)):
            yield f"layers.{i}.{name}", "norm", norm
    yield "norm", "norm", model.norm


def save_packed_weights(model: Any, path: str) -> None:
    """Cache a loaded model in its device layout (packed 2-bit ternary matrices,
    per-tensor scales, bf16 norms, the core-matrix-tiled embedding / lm_head) as
    one safetensors file, so that later loads skip quantisation and packing
    (load_packed_weights).  The layout is this library's; the file records the
    model shape and is rejected for any other."""
    from safetensors.torch import save_file

    tensors: dict[str, torch.Tensor] = {}
    meta: dict[str, Any] = {"format": _PACKED_FORMAT, "config": dict(vars(model.config)), "linears": {}}
    for name, kind, obj in _model_parts(model):
        if kind == "linear":
            tensors[name + ".packed"] = obj.weight.detach().cpu().contiguous()
            meta["linears"][name] = {"scale": obj.weight_scale, "segments": obj._segments}
        else:
            tensors[name + ".weight"] = obj.weight.detach().cpu().contiguous()
    tensors["embed_tokens.weight_tiled"] = model.embed_tokens.weight_tiled.detach().cpu().contiguous()
    tied = model.lm_head_tiled is model.embed_tokens.weight_tiled
    meta["tied_lm_head"] = tied
    if not tied:
        tensors["lm_head_tiled"] = model.lm_head_tiled.detach().cpu().contiguous()
    save_file(tensors, path, metadata={"bitnet": json.dumps(meta)})


def load_packed_weights(model: Any, path: str) -> None:
    """Load a save_packed_weights file into a model of the same shape: the device
    tensors are copied as they are (no quantisation, no packing kernels)."""
    from safetensors import safe_open

    with safe_open(path, framework="pt") as f:
        meta = json.loads((f.metadata() or {}).get("bitnet", "{}"))
        if meta.get("format") != _PACKED_FORMAT:
            raise ValueError(f"{path}: not a packed BitNet weight file")
        want = dict(vars(model.config))
        got = meta["config"]
        for key in ("hidden_size", "num_layers", "num_attention_heads", "num_key_value_heads", "intermediate_size",
                    "vocab_size", "head_dim"):
            if key in want and want.get(key) != got.get(key):
                raise ValueError(f"{path}: {key} {got.get(key)} does not match the model's {want.get(key)}")
        dev = model.device
        for name, kind, obj in _model_parts(model):
            if kind == "linear":
                obj.weight = f.get_tensor(name + ".packed").to(dev)
                info = meta["linears"][name]
                obj.weight_scale = float(info["scale"])
                obj._segments = [tuple(sg) for sg in info["segments"]] if info["segments"] else None
                obj._use_packed_ternary = True
            else:
                obj.weight = f.get_tensor(name + ".weight").to(dev)
        model.embed_tokens.weight_tiled = f.get_tensor("embed_tokens.weight_tiled").to(dev)
        model.lm_head_tiled = (model.embed_tokens.weight_tiled if meta.get("tied_lm_head")
                               else f.get_tensor("lm_head_tiled").to(dev))


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
