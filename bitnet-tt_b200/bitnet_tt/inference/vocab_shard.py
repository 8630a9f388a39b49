"""Vocabulary-sharded lm_head + argmax for batch-split multi-GPU decoding.

Each of the N ranks decodes its own sequences (batch split, replicated layer
weights, no collective in the layers).  Optionally the 128256-row lm_head is
split into N vocabulary shards, so that every rank reads 1/N of the 657 MB bf16
table per step instead of all of it.  One step of the head then is:

  1. all-gather of every rank's final-normed hidden rows       ([N*B, K] bf16)
  2. lm_head + per-row argmax over the local shard for all rows -> (value, global index)
  3. all-gather of the per-row pairs of all shards             ([N, N*B] pairs)
  4. merge of the N pairs of this rank's own rows -> next ids (+ positions advanced)

The merged ids equal the unsharded lm_head_argmax exactly: every logit is
computed by the same tile code, and the merge keeps the larger value, then the
smaller global index.  No counterpart exists in the reference (its lm_head runs
on one device, generator_batch32.py:768-811).

The collectives go through torch.distributed (NCCL over NVLink on GPUs, gloo in
the CPU tests); the device work is behind a small backend object so that the
protocol (shapes, shard bounds, gathers, merge, failures) is testable on CPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _lib

_PAIR_NONE = 0x7FFFFFFF  # index of "no row" pairs (value -inf)


def shard_bounds(vocab_size: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """(first tile, end tile, first row, row count) of rank's shard: whole 128-row
    tiles, the tiles split as evenly as possible, the last shard ragged."""
    ntiles = (vocab_size + 127) // 128
    per = (ntiles + world - 1) // world
    t0 = min(ntiles, rank * per)
    t1 = min(ntiles, t0 + per)
    r0 = t0 * 128
    rows = max(0, min(vocab_size, t1 * 128) - r0)
    return t0, t1, r0, rows


class CudaShardBackend:
    """Device work of the sharded head through the C ABI."""

    def shard_pairs(self, h: torch.Tensor, w_shard: torch.Tensor, rows: int, offset: int, ws: torch.Tensor,
                    pairs_out: torch.Tensor) -> None:
        if rows == 0:
            pairs_out[:, 0] = float("-inf")
            pairs_out[:, 1] = torch.tensor(_PAIR_NONE, dtype=torch.int32).view(torch.float32)
            return
        _lib.lm_head_argmax_shard(h, w_shard, rows, offset, ws, pairs_out)

    def merge(self, pairs: torch.Tensor, out_ids: torch.Tensor, positions: torch.Tensor | None) -> None:
        _lib.argmax_merge_pairs(pairs, out_ids, positions)

    def workspace(self, b: int, k: int, rows: int, device) -> torch.Tensor:
        return torch.zeros(max(1, _lib.argmax_workspace_bytes(b, k, max(rows, 1))), dtype=torch.uint8, device=device)


class VocabShardedLMHead:
    """The lm_head shard of this rank and the buffers of the four steps above.

    weight_tiled: the full tiled table (bitnet_pack_lm_head layout, uint8); the
    shard is a view of whole 128-row tiles of it (the tiles are contiguous).
    """

    def __init__(self, weight_tiled: torch.Tensor | None, vocab_size: int, hidden_size: int, batch: int,
                 device, group=None, backend=None) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.vocab_size, self.hidden_size, self.batch = vocab_size, hidden_size, batch
        self.device = torch.device(device)
        self.backend = backend if backend is not None else CudaShardBackend()
        t0, t1, self.offset, self.rows = shard_bounds(vocab_size, self.world, self.rank)
        tile_bytes = ((hidden_size + 7) // 8) * 2048
        self.shard = weight_tiled[t0 * tile_bytes:t1 * tile_bytes] if weight_tiled is not None else None
        n = self.world * batch
        self.gathered = torch.zeros((n, hidden_size), dtype=torch.bfloat16, device=self.device)
        self.pairs_local = torch.zeros((n, 2), dtype=torch.float32, device=self.device)
        self.pairs_all = torch.zeros((self.world, n, 2), dtype=torch.float32, device=self.device)
        self.own = torch.zeros((self.world, batch, 2), dtype=torch.float32, device=self.device)
        self.ws = self.backend.workspace(n, hidden_size, self.rows, self.device)

    def _all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(out, inp, group=self.group)
        else:
            parts = list(out.view(self.world, *inp.shape).unbind(0))
            dist.all_gather(parts, inp, group=self.group)

    def step(self, h_normed: torch.Tensor, out_ids: torch.Tensor, positions: torch.Tensor | None = None) -> None:
        """Next ids of this rank's rows from its final-normed hidden states."""
        if tuple(h_normed.shape) != (self.batch, self.hidden_size) or h_normed.dtype != torch.bfloat16:
            raise ValueError(f"hidden rows {tuple(h_normed.shape)} {h_normed.dtype}: expected "
                             f"({self.batch}, {self.hidden_size}) bfloat16")
        if out_ids.numel() != self.batch:
            raise ValueError("out_ids must hold one id per row")
        self._all_gather(self.gathered, h_normed.contiguous())
        self.backend.shard_pairs(self.gathered, self.shard, self.rows, self.offset, self.ws, self.pairs_local)
        self._all_gather(self.pairs_all, self.pairs_local)
        self.own.copy_(self.pairs_all[:, self.rank * self.batch:(self.rank + 1) * self.batch])
        self.backend.merge(self.own, out_ids, positions)
