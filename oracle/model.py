"""CPU oracle of the BitNet b1.58 decoder -- TEST INFRASTRUCTURE / CPU BASELINE ONLY.

Restates, in PyTorch on the CPU, the model the reference measures its TT path
against: HF BitNet (transformers models/bitnet/modeling_bitnet.py:44-261; decoder
layer order 232-261, attention 179-218, MLP 76-77, RMSNorm 53-58, half-split RoPE
89-110) with the reference's quantisers (src/bitnet_tt/utils/quantization.py:32-91:
ternary absmean weights, per-token int8 absmax activations) and the reference's
layer wiring (src/bitnet_tt/model/transformer.py:181-254, ffn.py:129-183,
attention.py:1040-1262).  Rounding points of every BitLinear follow
oracle/bitlinear.py (checked against it bit for bit in tests); attention runs in
fp32 and its output is rounded to bf16.

The ternary contraction is an fp32 matmul of integer-valued tensors: every
product and partial sum is an integer below 2^24, so it is exact in any order.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import quant as oq


def bf(x: torch.Tensor) -> torch.Tensor:
    """Round float32 to the bf16 grid (ties to even) and widen back."""
    return x.to(torch.bfloat16).to(torch.float32)


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor | None, eps: float) -> torch.Tensor:
    if gamma is None:
        return x
    k = x.shape[-1]
    ss = (x.double() ** 2).sum(-1, keepdim=True)
    var = (ss / k).float()
    r = 1.0 / torch.sqrt(var + torch.tensor(eps, dtype=torch.float32))
    return bf(gamma * bf(x * r))


def bitlinear(x: torch.Tensor, gamma: torch.Tensor | None, eps: float, w: torch.Tensor,
              col_scale: torch.Tensor) -> torch.Tensor:
    """Fused BitLinear on float32 tensors holding bf16 / ternary values.
    Returns bf16-valued float32 y = bf16(acc * (w_scale / s))."""
    a = rmsnorm(x, gamma, eps)
    amax = a.abs().amax(-1).clamp_min(torch.tensor(1e-5, dtype=torch.float32))
    s = torch.tensor(127.0, dtype=torch.float32) / amax
    q = torch.round(a * s[:, None]).clamp(-128, 127)
    acc = q @ w.t()
    return bf(acc * (col_scale[None, :] / s[:, None]))


def rope_tables(head_dim: int, max_len: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """HF BitNetRotaryEmbedding: cos/sin(pos * inv_freq) in fp32, cast to bf16."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    ang = torch.arange(max_len, dtype=torch.float32)[:, None] * inv_freq[None, :]
    return bf(torch.cos(ang)), bf(torch.sin(ang))


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., d] with cos/sin [..., d/2] broadcastable; HF apply_rotary_pos_emb in bf16 ops."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    o1 = bf(bf(x1 * cos) + bf(-x2 * sin))
    o2 = bf(bf(x2 * cos) + bf(x1 * sin))
    return torch.cat([o1, o2], dim=-1)


@dataclass
class OracleLayer:
    in_ln: torch.Tensor
    post_ln: torch.Tensor
    attn_ln: torch.Tensor
    ffn_ln: torch.Tensor
    w_qkv: torch.Tensor
    s_qkv: torch.Tensor
    w_o: torch.Tensor
    s_o: torch.Tensor
    w_g: torch.Tensor
    s_g: torch.Tensor
    w_u: torch.Tensor
    s_u: torch.Tensor
    w_d: torch.Tensor
    s_d: torch.Tensor


def _np(v) -> np.ndarray:
    if isinstance(v, torch.Tensor):
        return v.detach().float().cpu().numpy()
    return np.asarray(v, dtype=np.float32)


def _tern(w, quant: str = "numpy") -> tuple[torch.Tensor, float]:
    """Absmean ternary codes (as float32) and scale.  "numpy" is the reference
    quantiser bit for bit (quantization.py:32-57); "torch" evaluates the same
    formula with multi-threaded torch ops (the mean may differ in its last bit),
    used only where the oracle is timed rather than compared."""
    if quant == "torch":
        t = w if isinstance(w, torch.Tensor) else torch.from_numpy(np.asarray(w, np.float32))
        t = t.float()
        s = torch.clamp(t.abs().mean(), min=1e-5)
        return torch.clamp(torch.round(t / s), -1, 1), float(s)
    q, s = oq.weight_quant_ternary(_np(w))
    return torch.from_numpy(q.astype(np.float32)), float(s)


class OracleBitNet:
    """Greedy-decoding BitNet on the CPU from a (converted-key) state dict."""

    def __init__(self, config, state_dict, max_len: int = 2048, quant: str = "numpy"):
        self.cfg = config
        c = config
        self.d = c.head_dim
        self.nq, self.nkv = c.num_attention_heads, c.num_key_value_heads
        self.eps = c.rms_norm_eps
        t = lambda v: bf(v.float() if isinstance(v, torch.Tensor) else torch.from_numpy(_np(v)))  # noqa: E731
        self.embed = t(state_dict["embed_tokens.weight"])
        self.lm_head = t(state_dict["lm_head.weight"]) if "lm_head.weight" in state_dict else self.embed
        self.norm = t(state_dict["norm.weight"])
        self.layers: list[OracleLayer] = []
        for i in range(c.num_layers):
            p = f"layers.{i}."
            wq, sq = _tern(state_dict[p + "self_attn.q_proj.weight"], quant)
            wk, sk = _tern(state_dict[p + "self_attn.k_proj.weight"], quant)
            wv, sv = _tern(state_dict[p + "self_attn.v_proj.weight"], quant)
            wo, so = _tern(state_dict[p + "self_attn.o_proj.weight"], quant)
            wg, sg = _tern(state_dict[p + "mlp.gate_proj.weight"], quant)
            wu, su = _tern(state_dict[p + "mlp.up_proj.weight"], quant)
            wd, sd = _tern(state_dict[p + "mlp.down_proj.weight"], quant)
            s_qkv = torch.cat([torch.full((wq.shape[0],), sq), torch.full((wk.shape[0],), sk),
                               torch.full((wv.shape[0],), sv)]).float()
            self.layers.append(OracleLayer(
                in_ln=t(state_dict[p + "input_layernorm.weight"]), post_ln=t(state_dict[p + "post_attention_layernorm.weight"]),
                attn_ln=t(state_dict[p + "self_attn.attn_sub_norm.weight"]), ffn_ln=t(state_dict[p + "mlp.ffn_sub_norm.weight"]),
                w_qkv=torch.cat([wq, wk, wv]), s_qkv=s_qkv,
                w_o=wo, s_o=torch.full((wo.shape[0],), so), w_g=wg, s_g=torch.full((wg.shape[0],), sg),
                w_u=wu, s_u=torch.full((wu.shape[0],), su), w_d=wd, s_d=torch.full((wd.shape[0],), sd)))
        self.cos, self.sin = rope_tables(self.d, max_len, c.rope_theta)
        self.max_len = max_len

    def new_cache(self, batch: int) -> list[tuple[torch.Tensor, torch.Tensor]]:
        shape = (batch, self.nkv, self.max_len, self.d)
        return [(torch.zeros(shape), torch.zeros(shape)) for _ in self.layers]

    def attention(self, qkv: torch.Tensor, pos: torch.Tensor, cache) -> torch.Tensor:
        b = qkv.shape[0]
        d, nq, nkv = self.d, self.nq, self.nkv
        q = qkv[:, : nq * d].reshape(b, nq, d)
        k = qkv[:, nq * d:(nq + nkv) * d].reshape(b, nkv, d)
        v = qkv[:, (nq + nkv) * d:].reshape(b, nkv, d)
        cos, sin = self.cos[pos.long()][:, None, :], self.sin[pos.long()][:, None, :]
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        kc, vc = cache
        out = torch.empty(b, nq, d)
        g = nq // nkv
        for i in range(b):
            p = int(pos[i])
            kc[i, :, p] = k[i]
            vc[i, :, p] = v[i]
            keys, vals = kc[i, :, : p + 1], vc[i, :, : p + 1]           # [nkv, L, d]
            qi = q[i].reshape(nkv, g, d)
            sc = torch.einsum("hgd,hld->hgl", qi, keys) * (d ** -0.5)
            pr = torch.softmax(sc, dim=-1)
            out[i] = torch.einsum("hgl,hld->hgd", pr, vals).reshape(nq, d)
        return bf(out.reshape(b, nq * d))

    def prefill_attention(self, qkv: torch.Tensor, b: int, plen: int, cache) -> torch.Tensor:
        """Causal attention of b prompts of plen tokens at positions 0 .. plen-1
        (qkv [b*plen, (nq + 2 nkv) d]): the reference's prefill branch
        (src/bitnet_tt/layers/attention.py:1348-1507: RoPE over the prompt 1396,
        fill_cache_range 1411-1418, causal SDPA with scale d^-0.5 1465-1484).
        Writes cache rows 0 .. plen-1; returns bf16-valued [b*plen, nq d]."""
        d, nq, nkv = self.d, self.nq, self.nkv
        x = qkv.reshape(b, plen, -1)
        q = x[..., : nq * d].reshape(b, plen, nq, d)
        k = x[..., nq * d:(nq + nkv) * d].reshape(b, plen, nkv, d)
        v = x[..., (nq + nkv) * d:].reshape(b, plen, nkv, d)
        cos, sin = self.cos[:plen][None, :, None, :], self.sin[:plen][None, :, None, :]
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        kc, vc = cache
        kc[:, :, :plen] = k.permute(0, 2, 1, 3)
        vc[:, :, :plen] = v.permute(0, 2, 1, 3)
        g = nq // nkv
        qh = q.permute(0, 2, 1, 3).reshape(b, nkv, g, plen, d)
        sc = torch.einsum("bhgpd,bhld->bhgpl", qh, kc[:, :, :plen]) * (d ** -0.5)
        causal = torch.ones(plen, plen, dtype=torch.bool).triu(1)
        sc = sc.masked_fill(causal, float("-inf"))
        o = torch.einsum("bhgpl,bhld->bhgpd", torch.softmax(sc, dim=-1), vc[:, :, :plen])
        return bf(o.reshape(b, nq, plen, d).permute(0, 2, 1, 3).reshape(b * plen, nq * d))

    def prefill(self, prompts: np.ndarray, caches) -> tuple[torch.Tensor, torch.Tensor]:
        """All prompt tokens [B, L] in one batched pass (src/bitnet_tt/model/
        bitnet.py:217-313, mode "prefill"); fills cache rows 0 .. L-1 and returns
        (first generated ids [B], bf16-valued logits of the last prompt tokens)."""
        b, plen = prompts.shape
        h = self.embed[torch.from_numpy(prompts.reshape(-1).astype(np.int64))]
        for L, cache in zip(self.layers, caches):
            qkv = bitlinear(h, L.in_ln, self.eps, L.w_qkv, L.s_qkv)
            a = self.prefill_attention(qkv, b, plen, cache)
            h = bf(h + bitlinear(a, L.attn_ln, self.eps, L.w_o, L.s_o))
            n = rmsnorm(h, L.post_ln, self.eps)
            g = bitlinear(n, None, self.eps, L.w_g, L.s_g)
            u = bitlinear(n, None, self.eps, L.w_u, L.s_u)
            mid = bf(torch.where(g > 0, bf(g * g), torch.zeros_like(g)) * u)
            h = bf(h + bitlinear(mid, L.ffn_ln, self.eps, L.w_d, L.s_d))
        last = h.reshape(b, plen, -1)[:, -1]
        logits = bf(rmsnorm(last, self.norm, self.eps) @ self.lm_head.t())
        return torch.argmax(logits, dim=-1).to(torch.int32), logits

    def prefill_ragged(self, prompts: list[np.ndarray], caches) -> tuple[torch.Tensor, torch.Tensor]:
        """Prompts of different lengths: each sequence through prefill() on its
        own rows of the caches (the rows of one sequence never meet another's:
        per-token quantisation, attention within the sequence)."""
        ids, logits = [], []
        for b, p in enumerate(prompts):
            i, lg = self.prefill(np.asarray(p).reshape(1, -1), [(k[b:b + 1], v[b:b + 1]) for k, v in caches])
            ids.append(i)
            logits.append(lg)
        return torch.cat(ids), torch.cat(logits)

    def step(self, ids: torch.Tensor, pos: torch.Tensor, caches) -> tuple[torch.Tensor, torch.Tensor]:
        """One greedy decode step: (next ids [B], bf16-valued logits [B, V])."""
        h = self.embed[ids.long()]
        for L, cache in zip(self.layers, caches):
            qkv = bitlinear(h, L.in_ln, self.eps, L.w_qkv, L.s_qkv)
            a = self.attention(qkv, pos, cache)
            h = bf(h + bitlinear(a, L.attn_ln, self.eps, L.w_o, L.s_o))
            n = rmsnorm(h, L.post_ln, self.eps)
            g = bitlinear(n, None, self.eps, L.w_g, L.s_g)
            u = bitlinear(n, None, self.eps, L.w_u, L.s_u)
            mid = bf(torch.where(g > 0, bf(g * g), torch.zeros_like(g)) * u)
            h = bf(h + bitlinear(mid, L.ffn_ln, self.eps, L.w_d, L.s_d))
        normed = rmsnorm(h, self.norm, self.eps)
        logits = bf(normed @ self.lm_head.t())
        return torch.argmax(logits, dim=-1).to(torch.int32), logits

    def generate(self, prompts: np.ndarray, max_new_tokens: int) -> tuple[np.ndarray, list[torch.Tensor]]:
        """Equal-length prompts [B, L]: prompt tokens go through the decode step one
        at a time (as on the device); returns tokens [B, new] and per-step logits."""
        b, plen = prompts.shape
        caches = self.new_cache(b)
        pos = torch.zeros(b, dtype=torch.int32)
        ids = torch.from_numpy(prompts[:, 0].astype(np.int32))
        out, logits_all = [], []
        for t in range(plen + max_new_tokens - 1):
            nxt, logits = self.step(ids, pos, caches)
            pos = pos + 1
            if t + 1 < plen:
                ids = torch.from_numpy(prompts[:, t + 1].astype(np.int32))
            else:
                ids = nxt
                out.append(nxt.numpy())
                logits_all.append(logits)
        return np.stack(out, axis=1), logits_all
