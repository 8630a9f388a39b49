"""Pin of the model oracle (oracle/model.py) to the HF BitNet forward.

The reference checks its model against HF transformers' BitNet
(bench_accuracy.py:58-93 and examples/check_batch32_greedy_parity.py: HF
AutoModelForCausalLM is its accuracy oracle).  transformers is installed here
(models/bitnet/modeling_bitnet.py, integrations/bitnet.py), so this test builds
HF's BitNetForCausalLM on a small seeded configuration and compares it with the
oracle on the same weights:

  * every projection of HF's decoder is replaced by a linear layer whose weight
    is the ternary codes times their scale, as quantised ONCE by the reference's
    quantiser (src/bitnet_tt/utils/quantization.py:32-57) and shared with the
    oracle (HF's own WeightQuant multiplies by 1/s where the reference divides by
    s, which may round a tie the other way), and whose input goes through HF's
    own activation quantiser (integrations/bitnet.py ActQuant);
  * everything else is HF's code: embedding, RMSNorm placement (input, post-
    attention, attn_sub_norm before o_proj, ffn_sub_norm before down), half-split
    RoPE with theta 500000, grouped-query attention, ReLU^2 gate times up, the
    residual adds, the final norm and the tied lm_head.

Two comparisons, because a random-init BitNet is very sensitive to rounding:
one bf16 ulp of difference in a handful of attention outputs moves the int8
codes of the next BitLinear, and a 3-layer model's logits then move by 1-3%.

  * wiring (the pin): activation quantisation off on BOTH sides (HF linears
    without ActQuant, the oracle's BitLinears with act_quant=False), HF in
    float32.  The model is then smooth and only bf16-vs-float32 rounding is
    left (~1.5% on the logits); checked: last-token logits of a batched prefill
    and of 3 teacher-forced decode steps within WIRING_TOL, greedy ids equal
    except at near-ties.  Every planted wiring mistake in the oracle (on the
    CPU: skipped sub-norms or post-attention norm, interleaved GQA head groups,
    ReLU instead of ReLU^2, an untied head) moves the logits by more than
    5 x WIRING_TOL, so the bound separates correct from wrong wiring; RoPE,
    whose variants barely move the logits of short random prompts, is pinned
    directly against HF's apply_rotary_pos_emb;
  * quantised (HF's ActQuant and the reference quantiser on): HF in bf16 as the
    reference's greedy-parity check runs it (examples/check_batch32_greedy_parity.py),
    logits within QUANT_TOL and greedy ids mostly equal.
The quantiser itself is pinned separately (golden vectors of the reference's
quantization.py, and HF ActQuant against the oracle's codes below)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import quant as oq

WIRING_TOL = 3e-2
QUANT_TOL = 7e-2


def _cfg():
    from bitnet_tt.config import BitNetConfig

    return BitNetConfig(hidden_size=256, num_layers=3, num_attention_heads=4, num_key_value_heads=2,
                        intermediate_size=512, vocab_size=1000, max_position_embeddings=128)


class _SharedCodes(torch.nn.Module):
    """y = HF ActQuant(x) @ (codes * scale)^T (ActQuant skipped when act_quant is
    False), accumulated in float32 and cast to the model's dtype, as the
    reference's kernels accumulate a BitLinear in float32."""

    def __init__(self, latent: np.ndarray, act_quant: bool):
        super().__init__()
        q, s = oq.weight_quant_ternary(latent.astype(np.float32))
        self.w32 = torch.from_numpy(q.astype(np.float32) * np.float32(s))  # not a buffer: stays float32
        self.act_quant = act_quant

    def forward(self, x):
        from transformers.integrations.bitnet import ActQuant

        a = ActQuant.apply(x.float()) if self.act_quant else x.float()
        return torch.nn.functional.linear(a, self.w32).to(x.dtype)


def _hf_model(cfg, sd, act_quant: bool):
    from transformers import BitNetConfig as HFConfig
    from transformers import BitNetForCausalLM

    hc = HFConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
                  num_hidden_layers=cfg.num_layers, num_attention_heads=cfg.num_attention_heads,
                  num_key_value_heads=cfg.num_key_value_heads, hidden_act="relu2",
                  max_position_embeddings=cfg.max_position_embeddings, rms_norm_eps=cfg.rms_norm_eps,
                  tie_word_embeddings=True, rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta})
    hc._attn_implementation = "eager"
    m = BitNetForCausalLM(hc).float().eval()
    t = lambda k: torch.from_numpy(np.asarray(sd[k], dtype=np.float32))  # noqa: E731
    with torch.no_grad():
        m.model.embed_tokens.weight.copy_(t("embed_tokens.weight"))
        m.lm_head.weight = m.model.embed_tokens.weight  # tied head
        m.model.norm.weight.copy_(t("norm.weight"))
        for i, layer in enumerate(m.model.layers):
            p = f"layers.{i}."
            layer.input_layernorm.weight.copy_(t(p + "input_layernorm.weight"))
            layer.post_attention_layernorm.weight.copy_(t(p + "post_attention_layernorm.weight"))
            layer.self_attn.attn_sub_norm.weight.copy_(t(p + "self_attn.attn_sub_norm.weight"))
            layer.mlp.ffn_sub_norm.weight.copy_(t(p + "mlp.ffn_sub_norm.weight"))
            for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                setattr(layer.self_attn, name, _SharedCodes(sd[p + f"self_attn.{name}.weight"], act_quant))
            for name in ("gate_proj", "up_proj", "down_proj"):
                setattr(layer.mlp, name, _SharedCodes(sd[p + f"mlp.{name}.weight"], act_quant))
    return m


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def _compare(step, hf_logits, ref_logits, excused, tol):
    from parity_rules import within_logit_tol

    rel = _rel(hf_logits, ref_logits)
    assert rel < tol, f"step {step}: HF vs oracle logits rel err {rel:.3e}"
    hf_ids, ref_ids = hf_logits.argmax(-1), ref_logits.argmax(-1)
    for b in range(hf_ids.shape[0]):
        if int(hf_ids[b]) != int(ref_ids[b]):
            excused.append((step, b, within_logit_tol(ref_logits[b], int(hf_ids[b]))[0]))
    return rel


def _run_both(hf, oracle, prompts, tol, steps=3):
    """Prefill + teacher-forced decode steps on both; returns (rels, mismatches)."""
    batch, plen = prompts.shape
    excused, rels = [], []
    with torch.no_grad(), torch.compiler.set_stance("force_eager"):
        out = hf(input_ids=torch.from_numpy(prompts), use_cache=True)
        past = out.past_key_values
        caches = oracle.new_cache(batch)
        ref_ids, ref_logits = oracle.prefill(prompts, caches)
        rels.append(_compare(0, out.logits[:, -1].float(), ref_logits, excused, tol))
        pos = torch.full((batch,), plen, dtype=torch.int32)
        ids = ref_ids
        for t in range(1, steps + 1):  # teacher-forced: both take the oracle's ids
            out = hf(input_ids=ids.long()[:, None], past_key_values=past, use_cache=True)
            past = out.past_key_values
            nxt, ref_logits = oracle.step(ids, pos, caches)
            rels.append(_compare(t, out.logits[:, -1].float(), ref_logits, excused, tol))
            pos, ids = pos + 1, nxt
    return rels, excused


def _sd(cfg, seed):
    from bitnet_tt.utils.weights import synthetic_state_dict

    lazy = synthetic_state_dict(cfg, seed=seed)
    return {k: lazy[k].numpy() for k in lazy}


@pytest.mark.parametrize("batch,plen", [(4, 12), (2, 33)])
def test_oracle_wiring_matches_hf_bitnet_forward(batch, plen):
    cfg = _cfg()
    sd = _sd(cfg, batch * 100 + plen)
    hf = _hf_model(cfg, sd, act_quant=False)
    oracle = om.OracleBitNet(cfg, sd, max_len=cfg.max_position_embeddings, act_quant=False)
    prompts = np.random.default_rng(plen).integers(0, cfg.vocab_size, size=(batch, plen))
    rels, mism = _run_both(hf, oracle, prompts, WIRING_TOL)
    print(f"HF wiring pin: logits rel err per step {['%.2e' % r for r in rels]}, id mismatches {mism}")
    assert all(ok for _, _, ok in mism), f"id mismatches beyond near-ties: {mism}"
    assert len(mism) <= max(1, batch * 4 // 10)


def _interleaved_rope(x, cos, sin):
    """A planted mistake: RoPE over adjacent pairs (x[2i], x[2i+1]) instead of halves."""
    x1, x2 = x[..., 0::2], x[..., 1::2]
    o1, o2 = om.bf(om.bf(x1 * cos) + om.bf(-x2 * sin)), om.bf(om.bf(x2 * cos) + om.bf(x1 * sin))
    return torch.stack([o1, o2], dim=-1).reshape(x.shape)


class _InterleavedGroups(om.OracleBitNet):
    """A planted mistake: query head h reads KV head h % n_kv instead of h // group."""

    def _perm(self):
        g = self.nq // self.nkv
        return [(h % g) * self.nkv + h // g for h in range(self.nq)]

    def _swap(self, qkv, inverse=False):
        d, nq = self.d, self.nq
        perm = self._perm()
        if inverse:
            perm = [perm.index(i) for i in range(nq)]
        q = qkv[:, : nq * d].reshape(-1, nq, d)[:, perm].reshape(-1, nq * d)
        return torch.cat([q, qkv[:, nq * d:]], dim=1)

    def attention(self, qkv, pos, cache):
        return self._swap(super().attention(self._swap(qkv), pos, cache), inverse=True)

    def prefill_attention(self, qkv, b, plen, cache):
        return self._swap(super().prefill_attention(self._swap(qkv), b, plen, cache), inverse=True)


def test_hf_pin_detects_planted_wiring_mistakes(monkeypatch):
    """Each wiring mistake planted in the oracle (CPU only) moves the logits far
    beyond the bound that the correct oracle meets."""
    cfg = _cfg()
    sd = _sd(cfg, 412)
    hf = _hf_model(cfg, sd, act_quant=False)
    prompts = np.random.default_rng(12).integers(0, cfg.vocab_size, size=(4, 12))
    with torch.no_grad(), torch.compiler.set_stance("force_eager"):
        hf_logits = hf(input_ids=torch.from_numpy(prompts)).logits[:, -1].float()

    def rel_of(oracle):
        _, ref = oracle.prefill(prompts, oracle.new_cache(4))
        return _rel(hf_logits, ref)

    def fresh(cls=om.OracleBitNet):
        return cls(cfg, sd, max_len=cfg.max_position_embeddings, act_quant=False)

    good = rel_of(fresh())
    assert good < WIRING_TOL
    planted = {}
    for name, field in (("no attn_sub_norm", "attn_ln"), ("no ffn_sub_norm", "ffn_ln"),
                        ("no post_attention_layernorm", "post_ln")):
        o = fresh()
        for L in o.layers:
            setattr(L, field, None)
        planted[name] = rel_of(o)
    planted["interleaved GQA groups"] = rel_of(fresh(_InterleavedGroups))
    with monkeypatch.context() as m:
        m.setattr(om, "relu2_mul", lambda g, u: om.bf(torch.relu(g) * u))
        planted["ReLU instead of ReLU^2"] = rel_of(fresh())
    o = fresh()
    o.lm_head = o.embed.roll(1, dims=0)  # a head that is not the embedding table
    planted["untied lm_head"] = rel_of(o)
    print(f"correct wiring {good:.3e}; planted mistakes {planted}")
    for name, rel in planted.items():
        assert rel > 5 * WIRING_TOL, f"{name}: rel err {rel:.3e} not separated from the correct {good:.3e}"


def test_hf_rope_matches_oracle():
    """HF apply_rotary_pos_emb with its BitNetRotaryEmbedding tables (bf16, as the
    bf16 HF model runs it) against the oracle's RoPE on the same q / k rows at
    positions 0 .. 999: equal within one bf16 ulp; the adjacent-pair variant and
    another theta differ by O(1) (so the oracle's convention is the HF one)."""
    from transformers import BitNetConfig as HFConfig
    from transformers.models.bitnet.modeling_bitnet import BitNetRotaryEmbedding, apply_rotary_pos_emb

    n, heads, d = 1000, 4, 128
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, heads, n, d, generator=g).to(torch.bfloat16)
    k = torch.randn(1, heads, n, d, generator=g).to(torch.bfloat16)
    hc = HFConfig(hidden_size=heads * d, num_attention_heads=heads,
                  rope_parameters={"rope_type": "default", "rope_theta": 500000.0})
    cos, sin = BitNetRotaryEmbedding(hc)(q, torch.arange(n)[None])
    hq, hk = apply_rotary_pos_emb(q, k, cos, sin)
    oc, os_ = om.rope_tables(d, n, 500000.0)
    c, s = oc[None, None], os_[None, None]
    other = [t[None, None] for t in om.rope_tables(d, n, 10000.0)]
    for hf_x, x in ((hq, q), (hk, k)):
        ours = om.rope(x.float(), c, s)
        ulp = 2.0 ** (torch.floor(torch.log2(ours.abs().clamp_min(1e-30))) - 7)
        assert bool(((hf_x.float() - ours).abs() <= ulp).all())
        assert _rel(om.rope(x.float(), *other), hf_x.float()) > 0.1
        assert _rel(_interleaved_rope(x.float(), c, s), hf_x.float()) > 0.1


@pytest.mark.parametrize("batch,plen", [(4, 12), (2, 33)])
def test_oracle_quantised_forward_tracks_hf_bitnet(batch, plen):
    cfg = _cfg()
    sd = _sd(cfg, batch * 100 + plen)
    hf = _hf_model(cfg, sd, act_quant=True).to(torch.bfloat16)
    oracle = om.OracleBitNet(cfg, sd, max_len=cfg.max_position_embeddings)
    prompts = np.random.default_rng(plen).integers(0, cfg.vocab_size, size=(batch, plen))
    rels, mism = _run_both(hf, oracle, prompts, QUANT_TOL)
    print(f"HF quantised: logits rel err per step {['%.2e' % r for r in rels]}, id mismatches {mism}")
    assert len(mism) <= max(1, batch * 4 // 4)


def test_hf_norm_and_activation_quant_agree_with_oracle_pieces():
    """HF BitNetRMSNorm in bf16 equals the oracle's RMSNorm (same rounding points:
    normalise in float32, round to bf16, times gamma) up to one bf16 ulp, and HF
    ActQuant's fake-quantised values are the reference quantiser's codes / scale."""
    from transformers.integrations.bitnet import ActQuant
    from transformers.models.bitnet.modeling_bitnet import BitNetRMSNorm

    from oracle import bitlinear as ob

    g = torch.Generator().manual_seed(1)
    x = torch.randn(6, 256, generator=g).to(torch.bfloat16).float()
    gamma = (1 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16).float()
    ours = om.rmsnorm(x, gamma, 1e-5)
    with torch.no_grad():
        n16 = BitNetRMSNorm(256, eps=1e-5).to(torch.bfloat16)
        n16.weight.copy_(gamma.to(torch.bfloat16))
        hf16 = n16(x.to(torch.bfloat16)).float()
    ulp = 2.0 ** (torch.floor(torch.log2(ours.abs().clamp_min(1e-30))) - 7)
    assert bool(((hf16 - ours).abs() <= ulp).all())
    with torch.compiler.set_stance("force_eager"):
        fq = ActQuant.apply(x)
    q, s, _ = ob.act_quant(x.numpy())
    np.testing.assert_allclose(fq.numpy(), q.astype(np.float32) / s[:, None], rtol=1e-6, atol=0)
