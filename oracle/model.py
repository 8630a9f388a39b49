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
The square root and the divisions of the norm and the activation scale use
NumPy's IEEE operations: torch's CPU sqrt and its Python-scalar division are
not correctly rounded for every input, the kernels' __fsqrt_rn / __fdiv_rn are.

Pinned to the installed HF BitNet forward (tests/test_hf_pin.py): wiring with
the activation quantiser off on both sides, planted wiring mistakes rejected,
RoPE against HF's apply_rotary_pos_emb, norm and ActQuant piece by piece.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import quant as oq


def bf(x: torch.Tensor) -> torch.Tensor:
    """Round float32 to the bf16 grid (ties to even) and widen back."""
    return x.to(torch.bfloat16).to(torch.float32)


def _ieee_rsqrt(var: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 1 / sqrt(var + eps) with IEEE-rounded sqrt and division (NumPy).
    torch's CPU sqrt and its Python-scalar division are not correctly rounded
    for every input (measured: ~0.6% and ~25% of random float32 inputs differ
    by one ulp), while the kernels use __fsqrt_rn / __fdiv_rn."""
    v = var.numpy().astype(np.float32) + np.float32(eps)
    return torch.from_numpy(np.float32(1.0) / np.sqrt(v))


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor | None, eps: float) -> torch.Tensor:
    if gamma is None:
        return x
    k = x.shape[-1]
    ss = (x.double() ** 2).sum(-1, keepdim=True)
    var = (ss / k).float()
    r = _ieee_rsqrt(var, eps)
    return bf(gamma * bf(x * r))


def bitlinear(x: torch.Tensor, gamma: torch.Tensor | None, eps: float, w: torch.Tensor,
              col_scale: torch.Tensor, act_quant: bool = True) -> torch.Tensor:
    """Fused BitLinear on float32 tensors holding bf16 / ternary values.
    Returns bf16-valued float32 y = bf16(acc * (w_scale / s)).

    act_quant=False skips the int8 activation quantiser (y = bf16((a @ W^T) *
    w_scale) in float32): only the check of the decoder's wiring against the HF
    forward uses it, where the quantiser would turn bf16-vs-float32 rounding
    differences into code flips that mask what is compared."""
    a = rmsnorm(x, gamma, eps)
    wf = w if w.dtype == torch.float32 else w.float()  # int8-stored codes widen exactly
    if not act_quant:
        return bf((a @ wf.t()) * col_scale[None, :])
    amax = a.abs().amax(-1).clamp_min(torch.tensor(1e-5, dtype=torch.float32))
    s = torch.from_numpy(np.float32(127.0) / amax.numpy())  # IEEE division (see _ieee_rsqrt)
    q = torch.round(a * s[:, None]).clamp(-128, 127)
    acc = q @ wf.t()
    return bf(acc * (col_scale[None, :] / s[:, None]))


def relu2_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """HF BitNetMLP act_fn "relu2" (ReLU then square) times up, in bf16 steps."""
    return bf(torch.where(g > 0, bf(g * g), torch.zeros_like(g)) * u)


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

    # defaults for instances assembled field by field (attention-only checks)
    act_quant = True
    attn_dtype = torch.float32

    def __init__(self, config, state_dict, max_len: int = 2048, quant: str = "numpy", compact: bool = False,
                 act_quant: bool = True):
        """compact: keep the ternary codes as int8 (a quarter of the memory of the
        float32 codes; widened per use), for the full-depth 2B-4T-shaped model.
        act_quant=False: BitLinears without the activation quantiser (see
        bitlinear()); only for the wiring check against the HF forward."""
        self.cfg = config
        self.act_quant = act_quant
        # arithmetic of the attention's scores, softmax and weighted sum (the
        # output is rounded to bf16 either way); float64 gives a second, equally
        # valid reading of the fp32 attention, used to measure the noise floor
        self.attn_dtype = torch.float32
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
            if compact:
                wq, wk, wv, wo, wg, wu, wd = (w.to(torch.int8) for w in (wq, wk, wv, wo, wg, wu, wd))
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

    def new_cache(self, batch: int, length: int | None = None) -> list[tuple[torch.Tensor, torch.Tensor]]:
        shape = (batch, self.nkv, length or self.max_len, self.d)
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
            dt = self.attn_dtype
            keys, vals = kc[i, :, : p + 1].to(dt), vc[i, :, : p + 1].to(dt)  # [nkv, L, d]
            qi = q[i].reshape(nkv, g, d).to(dt)
            sc = torch.einsum("hgd,hld->hgl", qi, keys) * (d ** -0.5)
            pr = torch.softmax(sc, dim=-1)
            out[i] = torch.einsum("hgl,hld->hgd", pr, vals).reshape(nq, d).float()
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
        dt = self.attn_dtype
        qh = q.permute(0, 2, 1, 3).reshape(b, nkv, g, plen, d).to(dt)
        sc = torch.einsum("bhgpd,bhld->bhgpl", qh, kc[:, :, :plen].to(dt)) * (d ** -0.5)
        causal = torch.ones(plen, plen, dtype=torch.bool).triu(1)
        sc = sc.masked_fill(causal, float("-inf"))
        o = torch.einsum("bhgpl,bhld->bhgpd", torch.softmax(sc, dim=-1), vc[:, :, :plen].to(dt)).float()
        return bf(o.reshape(b, nq, plen, d).permute(0, 2, 1, 3).reshape(b * plen, nq * d))

    def layer(self, i: int, h: torch.Tensor, cache, attend) -> torch.Tensor:
        """Decoder layer i on hidden rows h (bf16-valued float32): input norm ->
        QKV -> attention (`attend(qkv, cache)`) -> attn_sub_norm -> o_proj +
        residual -> post-attention norm -> gate/up -> ReLU^2 * up ->
        ffn_sub_norm -> down + residual (HF modeling_bitnet.py:232-261, reference
        model/transformer.py:181-254)."""
        L, aq = self.layers[i], self.act_quant
        qkv = bitlinear(h, L.in_ln, self.eps, L.w_qkv, L.s_qkv, aq)
        a = attend(qkv, cache)
        h = bf(h + bitlinear(a, L.attn_ln, self.eps, L.w_o, L.s_o, aq))
        n = rmsnorm(h, L.post_ln, self.eps)
        g = bitlinear(n, None, self.eps, L.w_g, L.s_g, aq)
        u = bitlinear(n, None, self.eps, L.w_u, L.s_u, aq)
        mid = relu2_mul(g, u)
        return bf(h + bitlinear(mid, L.ffn_ln, self.eps, L.w_d, L.s_d, aq))

    def layer_prefill(self, i: int, h: torch.Tensor, b: int, plen: int, cache) -> torch.Tensor:
        """Layer i over the prompt rows h [b*plen, H]; writes cache rows 0 .. plen-1."""
        return self.layer(i, h, cache, lambda qkv, c: self.prefill_attention(qkv, b, plen, c))

    def layer_step(self, i: int, h: torch.Tensor, pos: torch.Tensor, cache) -> torch.Tensor:
        """Layer i for one decode token per sequence at positions pos; writes row pos."""
        return self.layer(i, h, cache, lambda qkv, c: self.attention(qkv, pos, c))

    def head(self, h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Final norm, tied lm_head and greedy argmax: (ids, bf16-valued logits)."""
        logits = bf(rmsnorm(h, self.norm, self.eps) @ self.lm_head.t())
        return torch.argmax(logits, dim=-1).to(torch.int32), logits

    def prefill(self, prompts: np.ndarray, caches) -> tuple[torch.Tensor, torch.Tensor]:
        """All prompt tokens [B, L] in one batched pass (src/bitnet_tt/model/
        bitnet.py:217-313, mode "prefill"); fills cache rows 0 .. L-1 and returns
        (first generated ids [B], bf16-valued logits of the last prompt tokens)."""
        b, plen = prompts.shape
        h = self.embed[torch.from_numpy(prompts.reshape(-1).astype(np.int64))]
        for i, cache in enumerate(caches):
            h = self.layer_prefill(i, h, b, plen, cache)
        return self.head(h.reshape(b, plen, -1)[:, -1])

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
        for i, cache in enumerate(caches):
            h = self.layer_step(i, h, pos, cache)
        return self.head(h)

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
