"""Token embedding tied to the lm_head (reference src/bitnet_tt/layers/embedding.py).

The bf16 table is stored once on the device, in the tiled layout the lm_head
kernel streams ([V/128][K/8][128 rows][8 bf16]); lookups gather from it.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _lib


class Embedding:
    def __init__(self, vocab_size: int, hidden_size: int, device=None) -> None:
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.device = torch.device(device if device is not None else "cuda")
        self.weight_tiled: torch.Tensor | None = None

    def load_weights(self, weight) -> None:
        if isinstance(weight, np.ndarray):
            weight = torch.from_numpy(np.ascontiguousarray(weight, dtype=np.float32))
        if tuple(weight.shape) != (self.vocab_size, self.hidden_size):
            raise ValueError(f"embedding shape {tuple(weight.shape)} != ({self.vocab_size}, {self.hidden_size})")
        w = weight.to(self.device).to(torch.bfloat16).contiguous()
        self.weight_tiled = _lib.pack_lm_head(w)

    def gather_into(self, ids: torch.Tensor, out: torch.Tensor) -> None:
        _lib.embed_gather(ids, self.weight_tiled, self.vocab_size, self.hidden_size, out)

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        ids32 = ids.reshape(-1).to(torch.int32).to(self.device).contiguous()
        out = torch.empty((ids32.numel(), self.hidden_size), dtype=torch.bfloat16, device=self.device)
        self.gather_into(ids32, out)
        return out.reshape(*ids.shape, self.hidden_size)
