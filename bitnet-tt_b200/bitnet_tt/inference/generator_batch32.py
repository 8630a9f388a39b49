"""Batched greedy decoding with the whole decode step captured in a CUDA graph.

Mirrors the reference's Batch32Generator (src/bitnet_tt/inference/generator_batch32.py:
__init__ 494-591, _decode_step_batch32 656-811, _capture_trace 1115-1181,
_execute_trace 1183-1195, generate_streaming 1597-1720).  Differences of
substance:
  * every row of the batch is a real sequence (the reference pads one user to
    32 rows), each with its own decode position, so the lm_head + argmax run
    on all rows;
  * one decode step is 9 kernels per layer + 4 (embedding gather, final norm,
    lm_head + argmax); its input (token ids) and position counters live on the
    device, the argmax kernel writes the next ids in place and advances the
    positions, so graph replays chain without host work;
  * prompts of one length go through a batched prefill (all B*L tokens per
    kernel: tcgen05 BitLinear tiles of 256 tokens, causal prompt attention),
    the reference's _prefill_batch32 (generator_batch32.py:1242-1279) without
    the copy into a separate batch-32 cache (1281-1353): the prefill writes
    the decode caches directly.  The part of a ragged prompt beyond the
    shortest one is consumed by the decode graph, one token per replay.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Iterator, Sequence

import numpy as np
import torch

from .. import _lib
from ..layers.attention import KVCache
from ..utils.rope import half_split_tables

PADDED_BATCH = 32


@dataclass
class GenerationStats:
    """reference generator_batch32.py:104-145."""

    prompt_tokens: int = 0
    generated_tokens: int = 0
    prefill_time: float = 0.0
    decode_time: float = 0.0
    step_times_ms: list[float] = field(default_factory=list)

    @property
    def ttft_ms(self) -> float:
        return self.prefill_time * 1000.0

    @property
    def tokens_per_second(self) -> float:
        return self.generated_tokens / self.decode_time if self.decode_time > 0 else 0.0

    @property
    def avg_ms_per_token(self) -> float:
        return 1000.0 * self.decode_time / max(1, len(self.step_times_ms))


class DecodeState:
    """Persistent device buffers of one batch (the graph's fixed addresses)."""

    def __init__(self, model, batch: int, max_seq_len: int, max_ctx: int = 0):
        cfg = model.config
        dev = model.device
        h, f = cfg.hidden_size, cfg.intermediate_size
        qkv = (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * cfg.head_dim
        self.batch, self.max_seq_len = batch, max_seq_len
        # bound on positions + 1 baked into the captured attention launches
        self.max_ctx = max_ctx or max_seq_len
        self.attn_ws = _lib.gqa_decode_workspace(batch, cfg.num_attention_heads, cfg.num_key_value_heads,
                                                 self.max_ctx, dev)
        self.ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.hidden = torch.zeros((batch, h), dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros((batch, qkv), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros((batch, cfg.num_attention_heads * cfg.head_dim), dtype=torch.bfloat16, device=dev)
        self.mid = torch.zeros((batch, f), dtype=torch.bfloat16, device=dev)
        self.normed = torch.zeros((batch, h), dtype=torch.bfloat16, device=dev)
        self.act_h = _lib.ActBuffers(batch, h, dev)
        self.act_f = _lib.ActBuffers(batch, f, dev)
        self.argmax_ws = torch.zeros(_lib.argmax_workspace_bytes(batch, h, cfg.vocab_size), dtype=torch.uint8,
                                     device=dev)
        self.caches = []
        for _ in range(cfg.num_layers):
            c = KVCache(max_seq_len, batch, cfg.num_key_value_heads, cfg.head_dim, dev)
            c.preallocate()
            self.caches.append(c)
        cos, sin = half_split_tables(cfg.head_dim, max_seq_len, cfg.rope_theta)
        self.rope_cos, self.rope_sin = cos.to(dev), sin.to(dev)
        self.logits: torch.Tensor | None = None
        self.plan: _lib.DecodePlan | None = None  # persistent all-layer launch (built outside capture)

    def kv_bytes(self) -> int:
        return sum(c.key_cache.numel() * 2 * 2 for c in self.caches)


class PrefillBuffers:
    """Activations of a batched prefill of `tokens` = B * L prompt tokens."""

    def __init__(self, model, tokens: int):
        cfg = model.config
        dev = model.device
        h, f = cfg.hidden_size, cfg.intermediate_size
        nq, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        self.tokens = tokens
        self.ids = torch.zeros(tokens, dtype=torch.int32, device=dev)
        self.hidden = torch.zeros((tokens, h), dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros((tokens, (nq + 2 * nkv) * d), dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros((tokens, nq * d), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros((tokens, nq * d), dtype=torch.bfloat16, device=dev)
        self.mid = torch.zeros((tokens, f), dtype=torch.bfloat16, device=dev)
        self.act_h = _lib.ActBuffers(tokens, h, dev)
        self.act_f = _lib.ActBuffers(tokens, f, dev)

    def nbytes(self) -> int:
        ts = [self.ids, self.hidden, self.qkv, self.q, self.attn, self.mid]
        for a in (self.act_h, self.act_f):
            ts += [a.q, a.row_scale, a.row_sum]
        return sum(t.numel() * t.element_size() for t in ts)


class Batch32Generator:
    def __init__(self, model, tokenizer: Any = None, enable_trace: bool = True, batch_size: int = PADDED_BATCH,
                 max_seq_len: int = 2048, keep_logits: bool = False, persistent: bool | None = None,
                 vocab_shard_group=None) -> None:
        self.model = model
        self.device = model.device
        self.config = model.config
        self.tokenizer = tokenizer
        self.enable_trace = enable_trace
        self.batch_size = batch_size
        self.max_seq_len = max_seq_len
        self.keep_logits = keep_logits
        self.state: DecodeState | None = None
        self._graph: torch.cuda.CUDAGraph | None = None
        # persistent=True: every layer in one launch (batch <= 32); default: 9 launches per layer
        self.persistent = bool(persistent) and batch_size <= PADDED_BATCH
        nl = self.config.num_layers
        # per layer: 4 fused BitLinear calls (1 launch each up to SIMT_FUSED_MAX_M tokens, else 2) + attention
        per_layer = 5 if batch_size <= _lib.SIMT_FUSED_MAX_M else 9
        self.launches_per_step = 6 if self.persistent else per_layer * nl + 5
        # vocab_shard_group: a torch.distributed group over which the lm_head is
        # split by vocabulary rows (batch-split multi-GPU decoding); its gathers
        # run outside the captured graph, after each replay
        self.vocab_shard_group = vocab_shard_group
        self.vocab_head = None
        if vocab_shard_group is not None:
            if keep_logits:
                raise ValueError("keep_logits is not available with a vocabulary-sharded lm_head")
            self.launches_per_step += 1  # shard lm_head: tile, GEMV, pairs, merge (final norm stays)
        self.last_stats = GenerationStats()
        self.context_limit = max_seq_len
        self.prefill_buffers: PrefillBuffers | None = None
        # batched_prefill=False: every prompt token goes through the decode graph
        self.batched_prefill = True
        self.prefill_chunk_tokens = 65536  # ragged prompts: tokens per prefill pass (bounds its buffers)
        # layer_probe(i, hidden): called with the hidden rows after the embedding
        # (i = -1) and after each layer i, from the eager paths only (prefill
        # passes, and decode steps with enable_trace=False); never inside a graph
        # capture.  Parity tests use it to compare every layer with the oracle.
        self.layer_probe = None

    def _probe(self, i: int, hidden: torch.Tensor) -> None:
        if self.layer_probe is not None and not torch.cuda.is_current_stream_capturing():
            self.layer_probe(i, hidden)

    def set_context_limit(self, n: int) -> None:
        """Bound the positions the next steps reach (positions + 1 <= n).  The
        attention sizes its grid by the limit in blocks of 256 keys, so the
        limit is rounded up to that; a new limit re-captures the decode graph."""
        n = min(self.max_seq_len, max(1, -(-int(n) // 256) * 256))
        if n != self.context_limit:
            self.context_limit = n
            self._graph = None
            if self.state is not None:
                st = self.state
                st.max_ctx = n
                st.plan = None
                st.attn_ws = _lib.gqa_decode_workspace(self.batch_size, self.config.num_attention_heads,
                                                       self.config.num_key_value_heads, n, self.device)

    # ---- state / graph -----------------------------------------------------
    def _ensure_state(self) -> DecodeState:
        if self.state is None:
            self.state = DecodeState(self.model, self.batch_size, self.max_seq_len, self.context_limit)
            if self.vocab_shard_group is not None:
                from .vocab_shard import VocabShardedLMHead

                m = self.model
                self.vocab_head = VocabShardedLMHead(m.lm_head_tiled, self.config.vocab_size, self.config.hidden_size,
                                                     self.batch_size, self.device, self.vocab_shard_group)
            if self.keep_logits:
                self.state.logits = torch.zeros((self.batch_size, self.config.vocab_size), dtype=torch.bfloat16,
                                                device=self.device)
        return self.state

    def _decode_step(self) -> None:
        """Enqueue one decode step on the current stream (graph-capturable)."""
        st = self.state
        m, cfg = self.model, self.config
        b, eps = st.batch, cfg.rms_norm_eps
        m.embed_tokens.gather_into(st.ids, st.hidden)
        self._probe(-1, st.hidden)
        if self.persistent:
            if st.plan is None:
                st.plan = _lib.DecodePlan(m, st.hidden, st.qkv, st.attn, st.mid, st.positions, st.rope_cos,
                                          st.rope_sin, st.caches, st.max_ctx, st.attn_ws)
            st.plan.run()
        # per layer: fused norm + act-quant + BitLinear calls (one launch each
        # below the ridge batch, act-quant + BitLinear above it) and the attention
        for i, (layer, cache) in enumerate(zip(m.layers, st.caches) if not self.persistent else ()):
            attn = layer.self_attn
            attn.qkv_proj.forward_fused(st.hidden, layer.input_layernorm.weight, eps, st.act_h, st.qkv)
            attn.decode_attention(st.qkv, st.positions, st.rope_cos, st.rope_sin, cache, st.attn, st.max_ctx,
                                  st.attn_ws)
            attn.o_proj.forward_fused(st.attn, attn.attn_sub_norm.weight, eps, st.act_h, st.hidden,
                                      residual=st.hidden)
            layer.mlp.gate_up_proj.forward_fused(st.hidden, layer.post_attention_layernorm.weight, eps, st.act_h,
                                                 st.mid)
            layer.mlp.down_proj.forward_fused(st.mid, layer.mlp.ffn_sub_norm.weight, eps, st.act_f, st.hidden,
                                              residual=st.hidden)
            self._probe(i, st.hidden)
        _lib.rmsnorm(st.hidden, m.norm.weight, eps, st.normed)
        if self.vocab_head is None:
            m.lm_head_argmax(st.normed, st.argmax_ws, st.ids, st.logits, st.positions)

    def _capture_trace(self) -> None:
        """Warm every kernel once eagerly, then capture the step into a CUDA graph."""
        st = self._ensure_state()
        saved_ids, saved_pos = st.ids.clone(), st.positions.clone()
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._decode_step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._decode_step()
        torch.cuda.synchronize(self.device)
        st.ids.copy_(saved_ids)
        st.positions.copy_(saved_pos)
        self._graph = g

    def release_trace(self) -> None:
        self._graph = None

    def step(self) -> None:
        """One decode step for the whole batch (graph replay or eager launches)."""
        if self.enable_trace:
            if self._graph is None:
                self._capture_trace()
            self._graph.replay()
        else:
            self._decode_step()
        if self.vocab_head is not None:
            st = self.state
            self.vocab_head.step(st.normed, st.ids, st.positions)

    def warmup(self) -> None:
        self._ensure_state()
        if self.enable_trace and self._graph is None:
            self._capture_trace()

    # ---- prompt processing ---------------------------------------------------
    def reset(self) -> None:
        st = self._ensure_state()
        st.positions.zero_()
        st.ids.zero_()

    def _prompts(self, input_ids) -> list[np.ndarray]:
        if isinstance(input_ids, torch.Tensor):
            input_ids = input_ids.cpu().numpy()
        if isinstance(input_ids, np.ndarray) and input_ids.ndim == 2:
            prompts = [np.asarray(r, dtype=np.int64) for r in input_ids]
        else:
            prompts = [np.asarray(p, dtype=np.int64).reshape(-1) for p in input_ids]
        if len(prompts) != self.batch_size:
            raise ValueError(f"{len(prompts)} prompts for a batch of {self.batch_size}")
        if any(p.size == 0 for p in prompts):
            raise ValueError("every prompt needs at least one token")
        if any(int(p.min()) < 0 or int(p.max()) >= self.config.vocab_size for p in prompts):
            raise ValueError("token id out of range")
        return prompts

    def release_prefill_buffers(self) -> None:
        self.prefill_buffers = None

    def _prefill_batched(self, table: np.ndarray) -> None:
        """All tokens of equal-length prompts table [B, L] in one pass per layer
        (reference model/bitnet.py:217-313, mode "prefill"); writes cache rows
        0 .. L-1 of every sequence, then the lm_head + argmax of the last
        tokens leaves the first generated ids in st.ids and L in st.positions.
        Enqueued on the current stream; the host does not wait."""
        st = self.state
        m, cfg = self.model, self.config
        b, plen = table.shape
        n = b * plen
        eps = cfg.rms_norm_eps
        nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        if self.prefill_buffers is None or self.prefill_buffers.tokens != n:
            self.prefill_buffers = None
            self.prefill_buffers = PrefillBuffers(m, n)
        pb = self.prefill_buffers
        pb.ids.copy_(torch.from_numpy(np.ascontiguousarray(table, dtype=np.int32).reshape(-1)))
        m.embed_tokens.gather_into(pb.ids, pb.hidden)
        self._probe(-1, pb.hidden)
        for i, (layer, cache) in enumerate(zip(m.layers, st.caches)):
            attn = layer.self_attn
            _lib.act_quant(pb.hidden, layer.input_layernorm.weight, eps, pb.act_h)
            attn.qkv_proj.forward_into(pb.act_h, n, pb.qkv)
            _lib.rope_append_prefill(pb.qkv, b, plen, nq, nkv, st.rope_cos, st.rope_sin, pb.q, cache.key_cache,
                                     cache.value_cache)
            _lib.attention_prefill(pb.q, cache.key_cache, cache.value_cache, b, plen, nq, nkv, attn.scale, pb.attn)
            _lib.act_quant(pb.attn, attn.attn_sub_norm.weight, eps, pb.act_h)
            attn.o_proj.forward_into(pb.act_h, n, pb.hidden, residual=pb.hidden)
            _lib.act_quant(pb.hidden, layer.post_attention_layernorm.weight, eps, pb.act_h)
            layer.mlp.gate_up_proj.forward_into(pb.act_h, n, pb.mid)
            _lib.act_quant(pb.mid, layer.mlp.ffn_sub_norm.weight, eps, pb.act_f)
            layer.mlp.down_proj.forward_into(pb.act_f, n, pb.hidden, residual=pb.hidden)
            self._probe(i, pb.hidden)
        last = pb.hidden.view(b, plen, -1)[:, plen - 1]  # row stride plen * hidden
        _lib.rmsnorm(last, m.norm.weight, eps, st.normed)
        st.positions.fill_(plen - 1)
        if self.vocab_head is None:
            m.lm_head_argmax(st.normed, st.argmax_ws, st.ids, st.logits, st.positions)
        else:
            self.vocab_head.step(st.normed, st.ids, st.positions)

    def _prefill_ragged(self, prompts: list[np.ndarray]) -> None:
        """Prompts of different lengths, packed without padding: sequences are
        taken in groups of at most `prefill_chunk_tokens` tokens (a longer
        prompt is a group of its own), and each group runs the prefill layers
        with the varlen RoPE / attention kernels (token offsets cu_seqlens) on
        its slice of the decode caches.  Then the final norm of every
        sequence's last prompt token and the lm_head + argmax leave the first
        generated ids in st.ids and each prompt's length in st.positions."""
        st = self.state
        m, cfg = self.model, self.config
        eps = cfg.rms_norm_eps
        nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        lens = [int(p.size) for p in prompts]
        groups, g0, tok = [], 0, 0
        for b, n in enumerate(lens):
            if b > g0 and tok + n > self.prefill_chunk_tokens:
                groups.append((g0, b))
                g0, tok = b, 0
            tok += n
        groups.append((g0, len(lens)))
        cap = max(sum(lens[a:e]) for a, e in groups)
        cap = cap if cap <= 256 else -(-cap // 256) * 256
        if self.prefill_buffers is None or self.prefill_buffers.tokens < cap:
            self.prefill_buffers = None
            self.prefill_buffers = PrefillBuffers(m, cap)
        pb = self.prefill_buffers
        last = torch.empty((len(lens), cfg.hidden_size), dtype=torch.bfloat16, device=self.device)
        for a, e in groups:
            glens = np.array(lens[a:e], dtype=np.int64)
            cu_h = np.zeros(e - a + 1, dtype=np.int32)
            cu_h[1:] = np.cumsum(glens)
            n = int(cu_h[-1])
            cu = torch.from_numpy(cu_h).to(self.device)
            pb.ids[:n].copy_(torch.from_numpy(np.concatenate(prompts[a:e]).astype(np.int32)))
            hidden, qkv, q, attn_out, mid = pb.hidden[:n], pb.qkv[:n], pb.q[:n], pb.attn[:n], pb.mid[:n]
            m.embed_tokens.gather_into(pb.ids[:n], hidden)
            self._probe(-1, hidden)
            lmax = int(glens.max())
            for i, (layer, cache) in enumerate(zip(m.layers, st.caches)):
                at = layer.self_attn
                kc, vc = cache.key_cache[a:e], cache.value_cache[a:e]
                _lib.act_quant(hidden, layer.input_layernorm.weight, eps, pb.act_h)
                at.qkv_proj.forward_into(pb.act_h, n, qkv)
                _lib.rope_append_prefill_varlen(qkv, cu, lmax, nq, nkv, st.rope_cos, st.rope_sin, q, kc, vc)
                _lib.attention_prefill_varlen(q, kc, vc, cu, lmax, nq, nkv, at.scale, attn_out)
                _lib.act_quant(attn_out, at.attn_sub_norm.weight, eps, pb.act_h)
                at.o_proj.forward_into(pb.act_h, n, hidden, residual=hidden)
                _lib.act_quant(hidden, layer.post_attention_layernorm.weight, eps, pb.act_h)
                layer.mlp.gate_up_proj.forward_into(pb.act_h, n, mid)
                _lib.act_quant(mid, layer.mlp.ffn_sub_norm.weight, eps, pb.act_f)
                layer.mlp.down_proj.forward_into(pb.act_f, n, hidden, residual=hidden)
                self._probe(i, hidden)
            last[a:e].copy_(hidden.index_select(0, cu[1:].long() - 1))
        _lib.rmsnorm(last, m.norm.weight, eps, st.normed)
        st.positions.copy_(torch.tensor(lens, dtype=torch.int32) - 1)
        if self.vocab_head is None:
            m.lm_head_argmax(st.normed, st.argmax_ws, st.ids, st.logits, st.positions)
        else:
            self.vocab_head.step(st.normed, st.ids, st.positions)

    def prefill(self, input_ids) -> np.ndarray:
        """Consume the prompts (ragged prompts allowed) in batched prefill
        passes: equal lengths as one [B, L] pass, different lengths packed
        (`_prefill_ragged`).  With batched_prefill = False every prompt token
        goes through the decode step instead.  Returns the prompt lengths;
        afterwards st.ids holds each sequence's first generated token and
        st.positions its next position."""
        prompts = self._prompts(input_ids)
        lens = np.array([p.size for p in prompts])
        if int(lens.max()) >= self.max_seq_len:
            raise ValueError("prompt longer than the KV cache")
        if int(lens.max()) > self.context_limit:
            self.set_context_limit(int(lens.max()))
        self.warmup()
        self.reset()
        st = self.state
        lmax, lmin = int(lens.max()), int(lens.min())
        if self.batched_prefill:
            if lmin == lmax:
                self._prefill_batched(np.stack(prompts))
            else:
                self._prefill_ragged(prompts)
            return lens
        # Token by token through the decode step.  A sequence whose prompt is
        # shorter than the longest one re-runs its last prompt token at its last
        # prompt position on every remaining step: that step rewrites the same
        # K/V row from the same inputs and produces the same first token, so when
        # the loop ends every sequence holds its first generated token and sits
        # at its own next position, as after the batched prefill.
        table = np.zeros((lmax, self.batch_size), dtype=np.int32)
        for b, p in enumerate(prompts):
            table[: p.size, b] = p
        table_d = torch.from_numpy(table).to(self.device)
        last_d = torch.from_numpy((lens - 1).astype(np.int64)).to(self.device)
        cols = torch.arange(self.batch_size, device=self.device)
        for t in range(lmax):
            idx = torch.clamp(last_d, max=t)  # per-sequence prompt index (and position) of this step
            st.ids.copy_(table_d[idx, cols])
            st.positions.copy_(idx.to(torch.int32))
            self.step()
        return lens

    # ---- generation ----------------------------------------------------------
    def generate(self, input_ids, max_new_tokens: int = 128) -> np.ndarray:
        """Greedy decode: returns [batch, max_new_tokens] token ids.  Prompts may
        differ in length (ragged prompts are prefilled packed, and every sequence
        continues from its own position)."""
        prompts = self._prompts(input_ids)
        lmax = max(p.size for p in prompts)
        if lmax + max_new_tokens > self.max_seq_len:
            raise ValueError("prompt + max_new_tokens exceeds the KV cache")
        stats = GenerationStats(prompt_tokens=int(sum(p.size for p in prompts)))
        self.set_context_limit(lmax + max_new_tokens)
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        self.prefill(prompts)
        out = torch.empty((max_new_tokens, self.batch_size), dtype=torch.int32, device=self.device)
        out[0].copy_(self.state.ids)
        torch.cuda.synchronize(self.device)
        t1 = time.perf_counter()
        for i in range(1, max_new_tokens):
            self.step()
            out[i].copy_(self.state.ids)
        torch.cuda.synchronize(self.device)
        t2 = time.perf_counter()
        stats.prefill_time, stats.decode_time = t1 - t0, t2 - t1
        stats.generated_tokens = (max_new_tokens - 1) * self.batch_size
        stats.step_times_ms = [1000.0 * (t2 - t1) / max(1, max_new_tokens - 1)] * max(0, max_new_tokens - 1)
        self.last_stats = stats
        return out.t().cpu().numpy()

    def generate_streaming(self, input_ids, max_new_tokens: int = 128) -> Iterator[np.ndarray]:
        """Yields each step's tokens [batch] on the host.  Every step copies the
        step's input ids from pinned host memory to the device and reads the new
        ids back (the reference's per-token H2D input copy and 4-byte readout,
        generator_batch32.py:1063-1083, 1355-1367)."""
        prompts = self._prompts(input_ids)
        self.set_context_limit(max(p.size for p in prompts) + max_new_tokens)
        self.prefill(prompts)
        host_in = torch.empty(self.batch_size, dtype=torch.int32, pin_memory=True)
        host_out = torch.empty(self.batch_size, dtype=torch.int32, pin_memory=True)
        host_out.copy_(self.state.ids)
        yield host_out.numpy().copy()
        for _ in range(1, max_new_tokens):
            host_in.copy_(host_out)
            self.state.ids.copy_(host_in, non_blocking=True)
            self.step()
            host_out.copy_(self.state.ids, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            yield host_out.numpy().copy()
