"""BitNet b1.58 model assembly (mirrors src/bitnet_tt/model/bitnet.py:33-365 of the reference).

create_model(config, device, weight_dtype="packed_ternary") builds the blocks;
load_weights_to_model (utils/weights.py) fills them.  The lm_head is tied to
the embedding table (BitNet-2B) unless a separate lm_head weight is loaded; it
stays bf16, as in HF, and is stored in the tiled layout its kernel streams.
"""

from __future__ import annotations

import torch

from .. import _lib
from ..config import BitNetConfig
from ..layers.bitlinear import RMSNorm
from ..layers.embedding import Embedding
from .transformer import TransformerBlock


class BitNetModel:
    def __init__(self, config: BitNetConfig, device=None, weight_dtype: str = "packed_ternary",
                 use_fused_rope: bool = True) -> None:
        self.config = config
        self.device = torch.device(device if device is not None else "cuda")
        self.embed_tokens = Embedding(config.vocab_size, config.hidden_size, self.device)
        self.layers = [TransformerBlock(config, self.device, i, weight_dtype, use_fused_rope)
                       for i in range(config.num_layers)]
        self.norm = RMSNorm(config.hidden_size, self.device, config.rms_norm_eps)
        self.lm_head_tiled: torch.Tensor | None = None

    # ---- loading (reference bitnet.py:93-137) ------------------------------
    def load_embedding_weights(self, weight) -> None:
        self.embed_tokens.load_weights(weight)

    def load_layer_weights(self, layer_idx: int, weights: dict) -> None:
        self.layers[layer_idx].load_weights(weights)

    def load_final_weights(self, norm_weight, lm_head_weight=None) -> None:
        self.norm.load_weights(norm_weight)
        if lm_head_weight is None:
            self.lm_head_tiled = self.embed_tokens.weight_tiled
        else:
            head = Embedding(self.config.vocab_size, self.config.hidden_size, self.device)
            head.load_weights(lm_head_weight)
            self.lm_head_tiled = head.weight_tiled

    # ---- eager forward of one decode step ----------------------------------
    def lm_head_argmax(self, hidden_normed: torch.Tensor, workspace: torch.Tensor, out_ids: torch.Tensor,
                       logits_out: torch.Tensor | None = None, advance_positions: torch.Tensor | None = None) -> None:
        _lib.lm_head_argmax(hidden_normed, self.lm_head_tiled, self.config.vocab_size, workspace, out_ids,
                            logits_out, advance_positions)

    def __call__(self, ids: torch.Tensor, positions: torch.Tensor, rope, caches, return_logits: bool = True):
        """Decode one token per sequence (eager).  Returns (next ids, logits | None)."""
        h = self.embed_tokens(ids.reshape(-1))
        for layer, cache in zip(self.layers, caches):
            h = layer(h, positions, rope, cache)
        normed = self.norm(h)
        b = normed.shape[0]
        ws = torch.empty(_lib.argmax_workspace_bytes(b, self.config.hidden_size, self.config.vocab_size), dtype=torch.uint8,
                         device=self.device)
        nxt = torch.empty(b, dtype=torch.int32, device=self.device)
        logits = (torch.empty((b, self.config.vocab_size), dtype=torch.bfloat16, device=self.device)
                  if return_logits else None)
        self.lm_head_argmax(normed, ws, nxt, logits)
        return nxt, logits


def create_model(config: BitNetConfig, device=None, weight_dtype: str = "packed_ternary",
                 use_fused_rope: bool = True) -> BitNetModel:
    """reference bitnet.py:364."""
    return BitNetModel(config, device, weight_dtype, use_fused_rope)
