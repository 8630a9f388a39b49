"""Vocabulary-sharded lm_head: the multi-rank protocol on CPU (gloo, 2 ranks).

The shard GEMV + argmax runs through a CPU stand-in backend here; the CUDA
kernels behind the real backend are checked against the unsharded lm_head in
tests/test_model_gpu.py.  Failures are made on the host: a rank that raises
before the gather, and a shape the head rejects before any collective.
"""

from __future__ import annotations

import datetime
import time
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest
import torch

V, K, B = 1000, 64, 4


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _table() -> torch.Tensor:
    g = torch.Generator().manual_seed(7)
    w = (0.05 * torch.randn((V, K), generator=g)).to(torch.bfloat16).float()
    w[123] = w[456]  # an exact tie between rows of different shards
    return w


class CpuBackend:
    """logits = bf16(h . W_shard^T); per row the best (value, global index), ties to the smaller index."""

    def __init__(self, w: torch.Tensor):
        self.w = w

    def workspace(self, b, k, rows, device):
        return torch.zeros(1)

    def shard_pairs(self, h, w_shard, rows, offset, ws, pairs_out):
        logits = (h.float() @ self.w[offset:offset + rows].t()).to(torch.bfloat16).float()
        v = logits.max(dim=1).values
        i = (logits == v[:, None]).int().argmax(dim=1) + offset
        pairs_out[:, 0] = v
        pairs_out[:, 1] = i.to(torch.int32).view(torch.float32)

    def merge(self, pairs, out_ids, positions):
        v = pairs[..., 0]
        idx = pairs[..., 1].contiguous().view(torch.int32)
        best_v = v.max(dim=0).values
        cand = torch.where(v == best_v[None, :], idx, torch.full_like(idx, 0x7FFFFFFF))
        out_ids.copy_(cand.min(dim=0).values)
        if positions is not None:
            positions += 1


def _worker(rank: int, world: int, port: int, mode: str, q) -> None:
    import torch.distributed as dist

    sys_path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "bitnet-tt_b200")
    import sys

    sys.path.insert(0, sys_path)
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        from bitnet_tt.inference.vocab_shard import VocabShardedLMHead, shard_bounds

        w = _table()
        head = VocabShardedLMHead(None, V, K, B, "cpu", backend=CpuBackend(w))
        g = torch.Generator().manual_seed(100 + rank)
        h = torch.randn((B, K), generator=g).to(torch.bfloat16)
        if rank == 0:
            h[0] = 0  # all logits 0: the whole vocabulary ties, the answer is row 0
        ids = torch.zeros(B, dtype=torch.int32)
        pos = torch.zeros(B, dtype=torch.int32)
        if mode == "shape":
            try:
                head.step(h[:, : K // 2].contiguous(), ids, pos)
                q.put((rank, "no error"))
            except ValueError:
                q.put((rank, "ValueError"))
            return
        if mode == "rank_fails" and rank == 1:
            q.put((rank, "raised"))
            raise SystemExit(3)  # leaves before the gather
        if mode == "stalls" and rank == 1:
            q.put((rank, ("stalled", time.time())))
            time.sleep(12)  # never reaches the gather in time; the peer's gather must end with an error
            return
        if mode == "fails_after":
            head.step(h, ids, pos)  # one complete step on both ranks
            if rank == 1:
                q.put((rank, "raised after a step"))
                raise SystemExit(3)
            t0 = time.time()
            try:
                head.step(h, ids, pos)
                q.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001 - the failure mode under test
                q.put((rank, (f"error: {type(e).__name__}", time.time() - t0)))
            return
        try:
            t0 = time.time()
            head.step(h, ids, pos)
        except Exception as e:  # noqa: BLE001 - the failure mode under test
            q.put((rank, f"error: {type(e).__name__}" if mode != "stalls" else
                   (f"error: {type(e).__name__}", time.time())))
            return
        logits = (h.float() @ w.t()).to(torch.bfloat16).float()
        ref = (logits == logits.max(dim=1).values[:, None]).int().argmax(dim=1).to(torch.int32)
        bounds = [shard_bounds(V, world, r) for r in range(world)]
        q.put((rank, {"ok": bool(torch.equal(ids, ref)), "pos": pos.tolist(), "ids": ids.tolist(),
                      "ref": ref.tolist(), "bounds": bounds}))
    except SystemExit:
        raise
    except Exception:  # noqa: BLE001
        q.put((rank, "exception: " + traceback.format_exc()))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(mode: str, world: int = 2, timeout: float = 60.0) -> dict:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_shard_bounds_cover_the_vocabulary():
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "bitnet-tt_b200"))
    from bitnet_tt.inference.vocab_shard import shard_bounds

    for v, world in [(1000, 2), (1000, 3), (128256, 8), (128256, 3), (100, 4)]:
        rows = [shard_bounds(v, world, r) for r in range(world)]
        covered = []
        for t0, t1, r0, n in rows:
            assert r0 % 128 == 0 and n >= 0
            covered += list(range(r0, r0 + n))
        assert covered == list(range(v))
    assert shard_bounds(128256, 8, 0)[3] == 126 * 128  # 1002 tiles -> 126 per rank, 120 on the last


def test_vocab_shard_two_ranks_matches_unsharded():
    out = _run("ok")
    for r in range(2):
        res = out[r]
        assert isinstance(res, dict), res
        assert res["ok"], res
        assert res["pos"] == [1] * B
    assert out[0]["ids"][0] == 0  # the all-tie row resolves to the smallest index


def test_vocab_shard_rank_failure_is_an_error_not_a_hang():
    out = _run("rank_fails")
    assert out[1] == "raised"
    assert isinstance(out[0], str) and out[0].startswith("error"), out[0]


def test_vocab_shard_rejects_wrong_hidden_width():
    out = _run("shape")
    assert out[0] == "ValueError" and out[1] == "ValueError"


def test_vocab_shard_rank_failure_after_a_step_is_an_error_not_a_hang():
    out = _run("fails_after")
    assert out[1] == "raised after a step"
    msg, waited = out[0]
    assert msg.startswith("error"), msg
    assert waited < 30.0  # the process-group timeout (5 s), not a hang


def test_vocab_shard_stalled_peer_times_out_with_an_error():
    """A rank that never reaches the gather: the other rank's gather ends with an
    error after the process-group timeout, while the staller is still asleep."""
    out = _run("stalls")
    state, t_stall = out[1]
    msg, t_err = out[0]
    assert state == "stalled" and msg.startswith("error"), (state, msg)
    assert t_err - t_stall < 12.0  # before the staller wakes up: a timeout, not a hang
