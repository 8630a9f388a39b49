"""CPU tests of the host-side code and of the oracle's internal consistency."""

import numpy as np
import pytest
import torch

from oracle import bitlinear as ob
from oracle import model as om
from oracle import quant as oq


def test_torch_oracle_bitlinear_equals_numpy_oracle():
    rng = np.random.default_rng(5)
    m, k, n = 7, 640, 200
    x = ob.round_bf16(rng.standard_normal((m, k)).astype(np.float32) * 3)
    g = ob.round_bf16((1 + 0.1 * rng.standard_normal(k)).astype(np.float32))
    w = rng.integers(-1, 2, size=(n, k)).astype(np.int8)
    ends, scales = [120, 160, 200], [0.02, 0.031, 0.0125]
    ref = ob.bitlinear(x, g, 1e-5, w, ends, scales)
    col = torch.from_numpy(ob.segment_scales(n, ends, scales))
    y = om.bitlinear(torch.from_numpy(x), torch.from_numpy(g), 1e-5, torch.from_numpy(w.astype(np.float32)), col)
    np.testing.assert_array_equal(y.numpy(), ref["y"])


def test_rope_tables_product_equals_oracle():
    import sys

    from bitnet_tt.utils.rope import half_split_tables

    cos, sin = half_split_tables(128, 4096, 500000.0)
    ocos, osin = om.rope_tables(128, 4096, 500000.0)
    np.testing.assert_array_equal(cos.float().numpy(), ocos.numpy())
    np.testing.assert_array_equal(sin.float().numpy(), osin.numpy())
    assert "bitnet_tt" in sys.modules


def test_reference_interleaved_rope_helper():
    from bitnet_tt.utils.rope import precompute_freqs_cis

    cos, sin = precompute_freqs_cis(64, 512)
    assert cos.shape == (1, 1, 512, 64) and sin.shape == (1, 1, 512, 64)
    assert np.all(np.abs(cos) <= 1) and np.all(np.abs(sin) <= 1)
    assert np.allclose(cos[..., 0::2], cos[..., 1::2])


def test_product_quantisers_match_oracle(golden):
    from bitnet_tt.utils import quantization as pq

    for name in ["wq_rand", "wq_large", "wq_zero", "wq_ties", "wq_odd"]:
        q, s = pq.weight_quant_ternary(golden[f"{name}_in"])
        np.testing.assert_array_equal(q, golden[f"{name}_q"])
        assert np.float32(s) == golden[f"{name}_s"]
    for name in ["aq_rand", "aq_zero", "aq_kat127", "aq_ties", "aq_large", "aq_tiny"]:
        q, s = pq.activation_quant_absmax(golden[f"{name}_in"])
        np.testing.assert_array_equal(q, golden[f"{name}_q"])
        np.testing.assert_array_equal(s.astype(np.float32), golden[f"{name}_s"])
    for name in ["pk_rand", "pk_odd", "pk_cfg0"]:
        packed = pq.pack_ternary_weights(golden[f"{name}_in"])
        np.testing.assert_array_equal(packed, golden[f"{name}_packed"])
        np.testing.assert_array_equal(pq.unpack_ternary_weights(packed, golden[f"{name}_in"].shape),
                                      golden[f"{name}_in"])


def test_gate_up_interleave_matches_oracle_row_order():
    from bitnet_tt.layers.ffn import interleave_gate_up

    f, h = 96, 8
    gate = torch.arange(f * h, dtype=torch.int32).reshape(f, h)
    up = -gate - 1
    fused = interleave_gate_up(gate, up)
    gr, ur = ob.fused_gate_up_rows(f)
    np.testing.assert_array_equal(fused[torch.from_numpy(gr)].numpy(), gate.numpy())
    np.testing.assert_array_equal(fused[torch.from_numpy(ur)].numpy(), up.numpy())


def test_fused_builders_keep_reference_contract():
    from bitnet_tt.layers.attention import build_fused_qkv_weight
    from bitnet_tt.layers.ffn import build_fused_gate_up_weight

    rng = np.random.default_rng(2)
    q, k, v = (rng.standard_normal(s).astype(np.float32) for s in [(64, 32), (16, 32), (16, 32)])
    fused, qs, ks, vs = build_fused_qkv_weight(q, k, v)
    assert fused.shape == (32, 96)
    np.testing.assert_array_equal(fused[:, :64], oq.weight_quant_ternary(q)[0].T)
    assert np.float32(ks) == np.float32(oq.weight_quant_ternary(k)[1])
    gu, gs, us = build_fused_gate_up_weight(q, q * 2)
    assert gu.shape == (32, 128) and np.isclose(us, 2 * gs)


def test_convert_hf_state_dict_and_layer_split():
    from bitnet_tt.utils.weights import convert_hf_state_dict, get_layer_weights

    hf = {"model.embed_tokens.weight": 1, "model.layers.0.input_layernorm.weight": 2, "model.norm.weight": 3,
          "lm_head.weight": 4, "model.layers.3.self_attn.q_proj.weight": 5, "model.rotary_emb.inv_freq": 6}
    c = convert_hf_state_dict(hf)
    assert c["embed_tokens.weight"] == 1 and c["norm.weight"] == 3 and c["lm_head.weight"] == 4
    assert c["layers.0.input_layernorm.weight"] == 2 and c["layers.3.self_attn.q_proj.weight"] == 5
    assert c["model.rotary_emb.inv_freq"] == 6  # unknown keys pass through unchanged
    assert get_layer_weights(c, 3) == {"self_attn.q_proj.weight": 5}


def test_synthetic_state_dict_is_deterministic():
    from bitnet_tt.config import BitNet2B4TConfig
    from bitnet_tt.utils.weights import synthetic_state_dict

    a = synthetic_state_dict(BitNet2B4TConfig(num_layers=2), seed=3)
    b = synthetic_state_dict(BitNet2B4TConfig(num_layers=2), seed=3)
    assert len(a) == 2 + 2 * 11
    k = "layers.1.self_attn.k_proj.weight"
    assert a[k].shape == (640, 2560)
    assert torch.equal(a[k], b[k])
    assert not torch.equal(a[k], synthetic_state_dict(BitNet2B4TConfig(num_layers=2), seed=4)[k])
    g = a["layers.0.input_layernorm.weight"]
    assert torch.equal(g, g.to(torch.bfloat16).float())


def test_configs_match_reference_defaults():
    from bitnet_tt.config import BitNet2B4TConfig, BitNetMiniConfig, get_config

    c = BitNet2B4TConfig()
    assert (c.hidden_size, c.num_layers, c.num_attention_heads, c.num_key_value_heads, c.intermediate_size,
            c.vocab_size, c.head_dim, c.rope_theta) == (2560, 30, 20, 5, 6912, 128256, 128, 500000.0)
    m = BitNetMiniConfig()
    assert (m.hidden_size, m.num_layers, m.num_attention_heads) == (256, 4, 4)
    assert isinstance(get_config("2b4t"), BitNet2B4TConfig)
    with pytest.raises(ValueError):
        get_config("nope")


def test_oracle_model_small_decode_runs():
    from bitnet_tt.config import BitNetConfig
    from bitnet_tt.utils.weights import synthetic_state_dict

    cfg = BitNetConfig(hidden_size=256, num_layers=2, num_attention_heads=2, num_key_value_heads=1,
                       intermediate_size=512, vocab_size=300)
    o = om.OracleBitNet(cfg, synthetic_state_dict(cfg, 1), max_len=32)
    prompts = np.random.default_rng(0).integers(0, 300, size=(3, 4))
    toks, logits = o.generate(prompts, 3)
    assert toks.shape == (3, 3) and len(logits) == 3
    assert toks.min() >= 0 and toks.max() < 300


def test_oracle_batched_prefill_equals_token_by_token():
    """The oracle's batched prefill (causal attention over the prompt) equals
    the prompt run through its decode step one token at a time: same caches,
    same last-token logits, same first ids (the orders of its fp32 sums do not
    reach the bf16 results on this case)."""
    import torch

    from bitnet_tt.config import BitNetConfig
    from bitnet_tt.utils.weights import synthetic_state_dict

    cfg = BitNetConfig(hidden_size=256, num_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       intermediate_size=512, vocab_size=300)
    o = om.OracleBitNet(cfg, synthetic_state_dict(cfg, 4), max_len=32)
    prompts = np.random.default_rng(2).integers(0, 300, size=(3, 9))
    caches = o.new_cache(3)
    ids, logits = o.prefill(prompts, caches)
    step_caches = o.new_cache(3)
    pos = torch.zeros(3, dtype=torch.int32)
    for t in range(prompts.shape[1]):
        nxt, step_logits = o.step(torch.from_numpy(prompts[:, t].astype(np.int32)), pos, step_caches)
        pos = pos + 1
    assert torch.equal(ids, nxt)
    assert torch.allclose(logits, step_logits, rtol=1e-2, atol=1e-2)
    for (k, v), (ks, vs) in zip(caches, step_caches):
        assert torch.allclose(k, ks, rtol=1e-2, atol=1e-2) and torch.allclose(v, vs, rtol=1e-2, atol=1e-2)


def test_hf_checkpoint_round_trip(tmp_path):
    """A synthetic checkpoint written in the HF layout (bf16 safetensors shards,
    HF key names, config.json) loads back through load_bitnet_weights with the
    reference's key conversion and config fields."""
    import torch

    from bitnet_tt.config import BitNetConfig
    from bitnet_tt.utils.weights import load_bitnet_weights, save_hf_checkpoint, synthetic_state_dict

    cfg = BitNetConfig(hidden_size=256, num_layers=2, num_attention_heads=2, num_key_value_heads=1,
                       intermediate_size=512, vocab_size=300, rms_norm_eps=1e-5)
    sd = synthetic_state_dict(cfg, 3)
    files = save_hf_checkpoint(sd, cfg, str(tmp_path), max_shard_bytes=300_000)
    assert len(files) > 1 and all(f.endswith(".safetensors") for f in files)
    sd2, cfg2 = load_bitnet_weights(str(tmp_path))
    assert sorted(sd2) == sorted(sd.keys())
    for k in sd.keys():
        ref = torch.as_tensor(np.asarray(sd[k], dtype=np.float32)).to(torch.bfloat16).float().numpy()
        np.testing.assert_array_equal(sd2[k], ref)
    for f in ("hidden_size", "num_layers", "num_attention_heads", "num_key_value_heads", "intermediate_size",
              "vocab_size", "rms_norm_eps", "rope_theta"):
        assert getattr(cfg2, f) == getattr(cfg, f), f
    assert "layers.1.self_attn.attn_sub_norm.weight" in sd2 and "embed_tokens.weight" in sd2


@pytest.mark.filterwarnings("ignore:overflow encountered")
@pytest.mark.parametrize("k", [2560, 6912])
def test_sum_of_squares_exact_span_and_extreme_rows(k):
    """Rows inside the documented span give the same fp64 sum of squares in every
    order (equal to the exact sum); rows far outside it may not, which is where
    device and oracle could stop agreeing bit for bit.  The oracle's quantiser
    stays finite on every extreme row (overflowing and underflowing variances)."""
    import math

    from extreme_rows import ROW_NAMES, extreme_rows, span_is_exact, var_orders

    rows = extreme_rows(k, seed=k)
    for name, row in zip(ROW_NAMES, rows):
        sq = row.astype(np.float64) ** 2
        if span_is_exact(row):
            assert float(np.sum(sq)) == math.fsum(sq.tolist()), name
            assert len(set(var_orders(row).values())) == 1, name
    assert span_is_exact(rows[1]) and not span_is_exact(rows[2])
    ref = ob.bitlinear(rows, np.ones(k, np.float32), 1e-5, np.zeros((1, k), np.int8))
    assert np.isfinite(ref["normed"]).all() and np.isfinite(ref["s"]).all()
    assert not ref["q"][4].any()  # var overflows fp32: r = 0, every normalised value 0, codes 0
