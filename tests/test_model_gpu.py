"""GPU parity of the supporting kernels and of the whole decode step against
the CPU oracle (through the product API, which calls the C ABI).

Tolerances: attention output within 2e-2 (fp32 softmax in a different order,
bf16 output); logits within 2e-2 relative (BASELINE); greedy tokens equal
except at documented near-ties: on identical inputs, top-2 oracle logits
within 2 bf16 ulps; after steps on the device's own KV cache (whose bf16
rows differ from the oracle's by rounding), the oracle logits of the two
tokens within the logits tolerance (2e-2 of the row's largest logit)."""

import numpy as np
import pytest
import torch

from oracle import bitlinear as ob
from oracle import model as om
from parity_rules import near_tie as _near_tie
from parity_rules import within_logit_tol as _within_logit_tol

pytestmark = pytest.mark.gpu


def _small_cfg(**kw):
    from bitnet_tt.config import BitNetConfig

    base = dict(hidden_size=512, num_layers=3, num_attention_heads=4, num_key_value_heads=2,
                intermediate_size=1024, vocab_size=1000, max_position_embeddings=256)
    base.update(kw)
    return BitNetConfig(**base)


def _numpy_sd(cfg, seed):
    from bitnet_tt.utils.weights import synthetic_state_dict

    sd = synthetic_state_dict(cfg, seed)
    return {k: sd[k].numpy() for k in sd}


def _device_model(cfg, sd, cuda):
    from bitnet_tt.model import create_model
    from bitnet_tt.utils.weights import load_weights_to_model

    m = create_model(cfg, cuda)
    load_weights_to_model(m, sd)
    return m


# ---------------------------------------------------------------------------
def _attention_case(cuda, b, nh, nkv, max_len, pos_list, max_ctx=0, seed=11):
    from bitnet_tt import _lib
    from bitnet_tt.utils.rope import half_split_tables

    d = 128
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn((b, (nh + 2 * nkv) * d), generator=g).to(torch.bfloat16)
    kc = torch.randn((b, nkv, max_len, d), generator=g).to(torch.bfloat16)
    vc = torch.randn((b, nkv, max_len, d), generator=g).to(torch.bfloat16)
    pos = torch.tensor(pos_list, dtype=torch.int32)
    cos, sin = half_split_tables(d, max_len, 500000.0)
    out = torch.empty((b, nh * d), dtype=torch.bfloat16, device=cuda)
    kd, vd = kc.to(cuda), vc.to(cuda)
    ws = _lib.gqa_decode_workspace(b, nh, nkv, max_ctx or max_len, cuda)
    _lib.gqa_decode_attention(qkv.to(cuda), nh, nkv, d, pos.to(cuda), cos.to(cuda), sin.to(cuda), kd, vd, d ** -0.5,
                              out, max_ctx, ws)
    torch.cuda.synchronize()
    assert _lib.last_device_status()[0] == 0
    if ws is not None:  # the kernel leaves its arrival counters at zero
        assert int(ws[: b * nkv * 4].view(torch.int32).abs().sum()) == 0

    o = om.OracleBitNet.__new__(om.OracleBitNet)
    o.d, o.nq, o.nkv = d, nh, nkv
    o.cos, o.sin = om.rope_tables(d, max_len, 500000.0)
    cache = (kc.float().clone(), vc.float().clone())
    ref = o.attention(qkv.float(), pos, cache)
    # appended rows: bit-exact (RoPE in bf16 ops, V copied)
    for i in range(b):
        p = int(pos[i])
        np.testing.assert_array_equal(kd[i, :, p].float().cpu().numpy(), cache[0][i, :, p].numpy())
        np.testing.assert_array_equal(vd[i, :, p].float().cpu().numpy(), cache[1][i, :, p].numpy())
    # the rest of the cache is untouched
    mask = torch.ones((b, max_len), dtype=torch.bool)
    mask[torch.arange(b), pos.long()] = False
    assert torch.equal(kd.cpu().permute(0, 2, 1, 3)[mask], kc.permute(0, 2, 1, 3)[mask])
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.numpy(), rtol=2e-2, atol=2e-2)


def test_attention_kernel_rope_append_and_softmax(cuda):
    _attention_case(cuda, 4, 20, 5, 300, [0, 7, 130, 299], max_ctx=300)


@pytest.mark.parametrize("nh,nkv", [(4, 4), (4, 2), (8, 2), (16, 2)])
def test_attention_group_sizes(cuda, nh, nkv):
    _attention_case(cuda, 3, nh, nkv, 200, [5, 16, 199], seed=nh * 10 + nkv)


def test_attention_split_context_ragged(cuda):
    # ragged contexts across several 256-key splits (config-4 style lengths)
    _attention_case(cuda, 6, 20, 5, 4096, [0, 255, 256, 1000, 2047, 4095], seed=3)


@pytest.mark.parametrize("b,max_len,units", [(32, 3000, 5), (150, 1024, 1)])
def test_attention_split_policy_long_units(cuda, b, max_len, units):
    # 32 x 3000 keys: five units of up to 608 keys per (sequence, KV head);
    # 150 x 1024: 750 (sequence, KV head) pairs fill the GPU, so one unit of up
    # to 1024 keys (16 tiles per warp) each
    from bitnet_tt import _lib

    want = 0 if units == 1 else 768 + b * 5 * units * (8 + 512) * 4
    assert _lib.gqa_decode_workspace_bytes(b, 20, 5, max_len) == want
    rng = np.random.default_rng(b)
    pos = sorted(rng.integers(0, max_len, size=b).tolist())
    pos[0], pos[1], pos[-1] = 0, 256, max_len - 1
    _attention_case(cuda, b, 20, 5, max_len, pos, seed=b)


def test_attention_split_repeated_calls(cuda):
    # the workspace counters must return to zero so that later calls merge correctly
    for rep in range(3):
        _attention_case(cuda, 2, 8, 2, 1024, [600 + rep, 1023 - rep], seed=20 + rep)


def test_attention_position_beyond_max_ctx_is_a_device_error(cuda):
    from bitnet_tt import _lib
    from bitnet_tt.utils.rope import half_split_tables

    b, nh, nkv, d, max_len = 2, 4, 2, 128, 512
    qkv = torch.zeros((b, (nh + 2 * nkv) * d), dtype=torch.bfloat16, device=cuda)
    kd = torch.zeros((b, nkv, max_len, d), dtype=torch.bfloat16, device=cuda)
    vd = torch.zeros_like(kd)
    cos, sin = half_split_tables(d, max_len, 500000.0)
    out = torch.empty((b, nh * d), dtype=torch.bfloat16, device=cuda)
    pos = torch.tensor([3, 300], dtype=torch.int32, device=cuda)
    # max_ctx 128: a single unit per (sequence, KV head), so no workspace
    _lib.gqa_decode_attention(qkv, nh, nkv, d, pos, cos.to(cuda), sin.to(cuda), kd, vd, 1.0, out, 128, None)
    torch.cuda.synchronize()
    code, site = _lib.last_device_status()
    assert code == -1 and site == 300  # a kernel bounds check reads back as BITNET_ERR_INVALID_ARGUMENT
    # a split context needs its workspace
    with pytest.raises(RuntimeError):
        _lib.gqa_decode_attention(qkv, nh, nkv, d, pos, cos.to(cuda), sin.to(cuda), kd, vd, 1.0, out, 512, None)


def _prefill_attention_case(cuda, b, plen, nh, nkv, max_len, seed=5):
    from bitnet_tt import _lib
    from bitnet_tt.utils.rope import half_split_tables

    d = 128
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn((b * plen, (nh + 2 * nkv) * d), generator=g).to(torch.bfloat16)
    kc = torch.randn((b, nkv, max_len, d), generator=g).to(torch.bfloat16)
    vc = torch.randn((b, nkv, max_len, d), generator=g).to(torch.bfloat16)
    cos, sin = half_split_tables(d, max_len, 500000.0)
    kd, vd = kc.to(cuda), vc.to(cuda)
    q = torch.empty((b * plen, nh * d), dtype=torch.bfloat16, device=cuda)
    out = torch.empty((b * plen, nh * d), dtype=torch.bfloat16, device=cuda)
    _lib.rope_append_prefill(qkv.to(cuda), b, plen, nh, nkv, cos.to(cuda), sin.to(cuda), q, kd, vd)
    _lib.attention_prefill(q, kd, vd, b, plen, nh, nkv, d ** -0.5, out)
    torch.cuda.synchronize()
    assert _lib.last_device_status()[0] == 0

    o = om.OracleBitNet.__new__(om.OracleBitNet)
    o.d, o.nq, o.nkv = d, nh, nkv
    o.cos, o.sin = om.rope_tables(d, max_len, 500000.0)
    cache = (kc.float().clone(), vc.float().clone())
    ref = o.prefill_attention(qkv.float(), b, plen, cache)
    # cache rows 0 .. plen-1 written bit-exactly (RoPE in bf16 ops, V copied), the rest untouched
    assert torch.equal(kd.float().cpu(), cache[0])
    assert torch.equal(vd.float().cpu(), cache[1])
    qr = om.rope(qkv.float()[:, : nh * d].reshape(b, plen, nh, d), o.cos[:plen][None, :, None], o.sin[:plen][None, :, None])
    assert torch.equal(q.float().cpu(), qr.reshape(b * plen, nh * d))
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.numpy(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("ragged", [False, True])
def test_rope_append_prefill_4byte_aligned_buffers_match(cuda, ragged):
    """Buffers that are 4- but not 16-byte aligned take the 4-byte kernel; 16-byte
    aligned ones the 16-byte kernel.  Both write identical queries and cache rows."""
    from bitnet_tt import _lib
    from bitnet_tt.utils.rope import half_split_tables

    b, plen, nh, nkv, max_len, d = 3, 37, 4, 2, 48, 128
    g = torch.Generator().manual_seed(21)
    qkv = torch.randn((b * plen, (nh + 2 * nkv) * d), generator=g).to(torch.bfloat16)
    cos, sin = half_split_tables(d, max_len, 500000.0)

    def offset_copy(t, off):  # same values at a data pointer 2 * off bytes past a 256-byte aligned base
        buf = torch.zeros(t.numel() + off, dtype=t.dtype, device=cuda)
        v = buf[off:].view(t.shape)
        v.copy_(t.to(cuda))
        return v

    results = []
    for off in (0, 2):
        args = [offset_copy(x, off) for x in (qkv, cos, sin)]
        q = offset_copy(torch.zeros((b * plen, nh * d), dtype=torch.bfloat16), off)
        kd = offset_copy(torch.zeros((b, nkv, max_len, d), dtype=torch.bfloat16), off)
        vd = offset_copy(torch.zeros((b, nkv, max_len, d), dtype=torch.bfloat16), off)
        assert (q.data_ptr() % 16 == 0) == (off == 0) and q.data_ptr() % 4 == 0
        if ragged:
            lens = [37, 5, 20]
            x = args[0][: sum(lens)]
            cu = torch.tensor([0, 37, 42, 62], dtype=torch.int32, device=cuda)
            _lib.rope_append_prefill_varlen(x, cu, max(lens), nh, nkv, args[1], args[2], q[: sum(lens)], kd, vd)
        else:
            _lib.rope_append_prefill(args[0], b, plen, nh, nkv, args[1], args[2], q, kd, vd)
        torch.cuda.synchronize()
        assert _lib.last_device_status()[0] == 0
        results.append((q.cpu(), kd.cpu(), vd.cpu()))
    for a, c in zip(*results):
        assert torch.equal(a, c)


@pytest.mark.parametrize("b,plen,nh,nkv,max_len", [
    (2, 150, 4, 2, 160),    # ragged last query / key block
    (1, 64, 8, 1, 64),      # group of 8 query heads, cache exactly the prompt
    (3, 1, 4, 4, 8),        # one-token prompts
    (1, 300, 20, 5, 512),   # BitNet-2B heads
    (2, 513, 2, 1, 600),    # key blocks past 8
])
def test_attention_prefill_matches_oracle(cuda, b, plen, nh, nkv, max_len):
    _prefill_attention_case(cuda, b, plen, nh, nkv, max_len, seed=b * 1000 + plen)


def test_attention_prefill_rejects_bad_arguments(cuda):
    from bitnet_tt import _lib

    kc = torch.zeros((1, 1, 16, 128), dtype=torch.bfloat16, device=cuda)
    q = torch.zeros((32, 256), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.attention_prefill(q, kc, kc, 1, 32, 2, 1, 0.1, q)  # prompt longer than the cache
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.attention_prefill(q, kc, kc, 2, 16, 3, 2, 0.1, q)  # heads not a multiple of kv heads


@pytest.mark.parametrize("batch,plen", [(4, 70), (32, 8)])
def test_batched_prefill_matches_oracle(cuda, batch, plen):
    """Generator prefill (all prompt tokens per kernel) against the oracle's
    batched prefill: first ids, logits of the last prompt tokens, KV caches."""
    from bitnet_tt.inference import Batch32Generator

    cfg = _small_cfg()
    sd = _numpy_sd(cfg, seed=21)
    model = _device_model(cfg, sd, cuda)
    prompts = np.random.default_rng(batch * plen).integers(0, cfg.vocab_size, size=(batch, plen))
    gen = Batch32Generator(model, batch_size=batch, max_seq_len=128, keep_logits=True)
    gen.prefill(prompts)
    assert gen.state.positions.cpu().tolist() == [plen] * batch
    dev_ids, dev_logits = gen.state.ids.cpu().numpy(), gen.state.logits.float().cpu()
    oracle = om.OracleBitNet(cfg, sd, max_len=128)
    caches = oracle.new_cache(batch)
    ref_ids, ref_logits = oracle.prefill(prompts, caches)
    rel = (dev_logits - ref_logits).norm() / ref_logits.norm()
    assert rel < 2e-2, f"logits rel err {rel:.3e}"
    assert not np.any((dev_ids != ref_ids.numpy()) & ~_near_tie(ref_logits).numpy())
    # layer 0 sees identical inputs: its keys and values are bit-exact
    c0 = gen.state.caches[0]
    assert torch.equal(c0.key_cache[:, :, :plen].float().cpu(), caches[0][0][:, :, :plen])
    assert torch.equal(c0.value_cache[:, :, :plen].float().cpu(), caches[0][1][:, :, :plen])
    for c, (kr, vr) in zip(gen.state.caches, caches):
        for dev, ref in ((c.key_cache, kr), (c.value_cache, vr)):
            d = dev[:, :, :plen].float().cpu()
            assert (d - ref[:, :, :plen]).norm() / ref[:, :, :plen].norm() < 2e-2


@pytest.mark.parametrize("chunk", [20, 65536, 0])
def test_ragged_prompts_prefill_matches_oracle(cuda, chunk):
    """Ragged prompts packed without padding (varlen RoPE / attention; chunk 20
    splits the batch into several prefill passes) against the oracle prefilling
    each sequence on its own; then decode steps at the sequences' own positions.
    chunk 0: batched_prefill = False, every prompt token through the decode
    step (short prompts re-run their last token while the longest finishes)."""
    from bitnet_tt.inference import Batch32Generator

    cfg = _small_cfg()
    sd = _numpy_sd(cfg, seed=5)
    model = _device_model(cfg, sd, cuda)
    rng = np.random.default_rng(3)
    lens = [5, 12, 9, 1, 17, 6, 70, 8]
    prompts = [rng.integers(0, cfg.vocab_size, size=n) for n in lens]
    gen = Batch32Generator(model, batch_size=len(lens), max_seq_len=96, keep_logits=True)
    gen.prefill_chunk_tokens = chunk or 65536
    gen.batched_prefill = chunk != 0
    gen.prefill(prompts)
    assert gen.state.positions.cpu().tolist() == lens
    ids, logits = [gen.state.ids.cpu().numpy().copy()], [gen.state.logits.float().cpu().clone()]
    for _ in range(3):
        gen.step()
        ids.append(gen.state.ids.cpu().numpy().copy())
        logits.append(gen.state.logits.float().cpu().clone())
    assert gen.state.positions.cpu().tolist() == [n + 3 for n in lens]
    dev_ids = np.stack(ids, 1)
    gen2 = Batch32Generator(model, batch_size=len(lens), max_seq_len=96)
    gen2.prefill_chunk_tokens = chunk or 65536
    gen2.batched_prefill = chunk != 0
    np.testing.assert_array_equal(gen2.generate(prompts, 4), dev_ids)  # the same through generate()

    oracle = om.OracleBitNet(cfg, sd, max_len=96)
    caches = oracle.new_cache(len(lens))
    ref_first, ref_logits0 = oracle.prefill_ragged(prompts, caches)
    c0 = gen.state.caches[0]
    for b, n in enumerate(lens):  # layer 0 sees identical inputs: its K/V rows are bit-exact
        assert torch.equal(c0.key_cache[b, :, :n].float().cpu(), caches[0][0][b, :, :n])
        assert torch.equal(c0.value_cache[b, :, :n].float().cpu(), caches[0][1][b, :, :n])
    rel = (logits[0] - ref_logits0).norm() / ref_logits0.norm()
    assert rel < 2e-2, f"logits rel err {rel:.3e}"
    ref_ids, ref_logits = [ref_first.numpy()], [ref_logits0]
    pos = torch.tensor(lens, dtype=torch.int32)
    cur = ref_first
    for _ in range(3):
        cur, lg = oracle.step(cur, pos, caches)
        pos = pos + 1
        ref_ids.append(cur.numpy())
        ref_logits.append(lg)
    ref_ids = np.stack(ref_ids, 1)
    for b in range(len(lens)):
        for t in range(dev_ids.shape[1]):
            if dev_ids[b, t] != ref_ids[b, t]:
                ok, why = _within_logit_tol(ref_logits[t][b], int(dev_ids[b, t]))
                assert ok, f"seq {b} step {t}: not a near-tie ({why})"
                break


def test_attention_prefill_varlen_matches_oracle(cuda):
    """Varlen RoPE / K-V append and causal attention on packed ragged prompts
    against the oracle's prefill attention of each sequence alone."""
    from bitnet_tt import _lib
    from bitnet_tt.utils.rope import half_split_tables

    lens = [1, 70, 129, 64, 300, 2]
    nh, nkv, d, max_len = 8, 2, 128, 320
    b = len(lens)
    cu_h = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    n = int(cu_h[-1])
    g = torch.Generator().manual_seed(23)
    qkv = torch.randn((n, (nh + 2 * nkv) * d), generator=g).to(torch.bfloat16)
    kc = torch.randn((b, nkv, max_len, d), generator=g).to(torch.bfloat16)
    vc = torch.randn((b, nkv, max_len, d), generator=g).to(torch.bfloat16)
    cos, sin = half_split_tables(d, max_len, 500000.0)
    kd, vd = kc.to(cuda), vc.to(cuda)
    q = torch.empty((n, nh * d), dtype=torch.bfloat16, device=cuda)
    out = torch.empty((n, nh * d), dtype=torch.bfloat16, device=cuda)
    cu = torch.from_numpy(cu_h).to(cuda)
    _lib.rope_append_prefill_varlen(qkv.to(cuda), cu, max(lens), nh, nkv, cos.to(cuda), sin.to(cuda), q, kd, vd)
    _lib.attention_prefill_varlen(q, kd, vd, cu, max(lens), nh, nkv, d ** -0.5, out)
    torch.cuda.synchronize()
    assert _lib.last_device_status()[0] == 0
    o = om.OracleBitNet.__new__(om.OracleBitNet)
    o.d, o.nq, o.nkv = d, nh, nkv
    o.cos, o.sin = om.rope_tables(d, max_len, 500000.0)
    kr, vr = kc.float().clone(), vc.float().clone()
    for i, L in enumerate(lens):
        ref = o.prefill_attention(qkv.float()[cu_h[i]:cu_h[i + 1]], 1, L, (kr[i:i + 1], vr[i:i + 1]))
        np.testing.assert_allclose(out[cu_h[i]:cu_h[i + 1]].float().cpu().numpy(), ref.numpy(), rtol=2e-2, atol=2e-2)
    assert torch.equal(kd.float().cpu(), kr) and torch.equal(vd.float().cpu(), vr)  # rows beyond each length untouched


def test_full_width_prefill_matches_oracle(cuda):
    """2B-4T widths, 2 layers, 4 prompts of 512 tokens (2048 prompt tokens:
    8 BitLinear token tiles, 8 key blocks per sequence)."""
    from bitnet_tt.config import BitNet2B4TConfig
    from bitnet_tt.inference import Batch32Generator

    cfg = BitNet2B4TConfig(num_layers=2, max_position_embeddings=1024)
    sd = _numpy_sd(cfg, seed=77)
    model = _device_model(cfg, sd, cuda)
    prompts = np.random.default_rng(9).integers(0, cfg.vocab_size, size=(4, 512))
    gen = Batch32Generator(model, batch_size=4, max_seq_len=576, keep_logits=True)
    gen.prefill(prompts)
    dev_logits = gen.state.logits.float().cpu()
    oracle = om.OracleBitNet(cfg, sd, max_len=576)
    ref_ids, ref_logits = oracle.prefill(prompts, oracle.new_cache(4))
    rel = (dev_logits - ref_logits).norm() / ref_logits.norm()
    assert rel < 2e-2, f"logits rel err {rel:.3e}"
    mismatch = gen.state.ids.cpu().numpy() != ref_ids.numpy()
    assert not np.any(mismatch & ~_near_tie(ref_logits).numpy())


def test_lm_head_argmax_and_embedding(cuda):
    from bitnet_tt import _lib

    b, k, v = 32, 2560, 1000
    g = torch.Generator().manual_seed(5)
    h = torch.randn((b, k), generator=g).to(torch.bfloat16)
    e = (0.02 * torch.randn((v, k), generator=g)).to(torch.bfloat16)
    tiled = _lib.pack_lm_head(e.to(cuda))
    np.testing.assert_array_equal(tiled.cpu().numpy().view(np.uint16),
                                  ob.lm_head_pack(e.view(torch.int16).numpy().view(np.uint16)))
    ids = torch.tensor([0, 5, 999, 128, 127, 500] + [3] * 26, dtype=torch.int32, device=cuda)
    emb = torch.empty((b, k), dtype=torch.bfloat16, device=cuda)
    _lib.embed_gather(ids, tiled, v, k, emb)
    np.testing.assert_array_equal(emb.cpu().view(torch.int16).numpy(), e[ids.cpu().long()].view(torch.int16).numpy())

    ws = torch.empty(_lib.argmax_workspace_bytes(b, k, v), dtype=torch.uint8, device=cuda)
    out = torch.empty(b, dtype=torch.int32, device=cuda)
    logits = torch.empty((b, v), dtype=torch.bfloat16, device=cuda)
    pos = torch.arange(b, dtype=torch.int32, device=cuda)
    _lib.lm_head_argmax(h.to(cuda), tiled, v, ws, out, logits, pos)
    torch.cuda.synchronize()
    ref = om.bf(h.float() @ e.float().t())
    got = logits.float().cpu()
    np.testing.assert_allclose(got.numpy(), ref.numpy(), rtol=2e-2, atol=1e-2)
    # the chosen id is the first maximum of the device's own bf16 logits ...
    assert torch.equal(out.cpu().long(), torch.argmax(got, dim=-1))
    # ... and an oracle maximum up to one bf16 ulp (near-ties)
    ulp = 2.0 ** (torch.floor(torch.log2(ref.abs().amax(-1))) - 7)
    chosen = ref.gather(1, out.cpu().long()[:, None])[:, 0]
    assert torch.all(ref.amax(-1) - chosen <= ulp)
    assert torch.equal(pos.cpu(), torch.arange(b, dtype=torch.int32) + 1)


def test_linear_api_bit_exact(cuda):
    from bitnet_tt.layers.bitlinear import Linear

    rng = np.random.default_rng(9)
    w = (0.02 * rng.standard_normal((384, 640))).astype(np.float32)
    x = torch.randn((5, 640), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(640, generator=torch.Generator().manual_seed(2))).to(torch.bfloat16)
    lin = Linear(640, 384, cuda, weight_dtype="packed_ternary")
    with pytest.raises(RuntimeError, match="Weights not loaded"):
        lin(x.to(cuda))
    lin.load_weights(w)
    y = lin(x.to(cuda), norm_weight=gamma.to(cuda), norm_epsilon=1e-5)
    from oracle import quant as oq

    wq, ws = oq.weight_quant_ternary(w)
    ref = ob.bitlinear(x.float().numpy(), gamma.float().numpy(), 1e-5, wq, [384], [float(ws)])
    np.testing.assert_array_equal(y.float().cpu().numpy(), ref["y"])
    with pytest.raises(ValueError):
        Linear(640, 384, cuda, weight_dtype="bfp4")


@pytest.mark.parametrize("batch", [4, 32])
def test_small_model_decode_matches_oracle(cuda, batch):
    from bitnet_tt.inference import Batch32Generator

    cfg = _small_cfg()
    sd = _numpy_sd(cfg, seed=7)
    model = _device_model(cfg, sd, cuda)
    prompts = np.random.default_rng(batch).integers(0, cfg.vocab_size, size=(batch, 8))
    new = 6
    gen = Batch32Generator(model, batch_size=batch, max_seq_len=64, keep_logits=True)
    gen.prefill(prompts)
    dev_tokens, dev_logits = [gen.state.ids.cpu().numpy().copy()], [gen.state.logits.float().cpu().clone()]
    for _ in range(new - 1):
        gen.step()
        dev_tokens.append(gen.state.ids.cpu().numpy().copy())
        dev_logits.append(gen.state.logits.float().cpu().clone())
    dev_tokens = np.stack(dev_tokens, axis=1)

    oracle = om.OracleBitNet(cfg, sd, max_len=64)
    ref_tokens, ref_logits = oracle.generate(prompts, new)
    # first step: same inputs on both sides
    rel = (dev_logits[0] - ref_logits[0]).norm() / ref_logits[0].norm()
    assert rel < 2e-2, f"logits rel err {rel:.3e}"
    # while the sequences agree, every step's logits (over those rows) are within tolerance
    agree = np.ones(batch, dtype=bool)
    for t in range(new):
        rows = torch.from_numpy(np.nonzero(agree)[0])
        if rows.numel():
            d, r = dev_logits[t][rows], ref_logits[t][rows]
            rr = (d - r).norm() / r.norm()
            assert rr < 2e-2, f"step {t}: logits rel err {rr:.3e} over {rows.numel()} agreeing rows"
        agree &= dev_tokens[:, t] == ref_tokens[:, t]
    for b in range(batch):
        for t in range(new):
            if dev_tokens[b, t] != ref_tokens[b, t]:
                ok, why = _within_logit_tol(ref_logits[t][b], int(dev_tokens[b, t]))
                assert ok, f"seq {b} step {t}: not a near-tie ({why})"
                break  # the sequences legitimately diverge after a near-tie


def test_graph_replay_equals_eager(cuda):
    from bitnet_tt.inference import Batch32Generator

    cfg = _small_cfg(num_layers=2)
    sd = _numpy_sd(cfg, seed=3)
    model = _device_model(cfg, sd, cuda)
    prompts = np.random.default_rng(1).integers(0, cfg.vocab_size, size=(32, 5))
    eager = Batch32Generator(model, batch_size=32, max_seq_len=32, enable_trace=False).generate(prompts, 8)
    traced = Batch32Generator(model, batch_size=32, max_seq_len=32, enable_trace=True).generate(prompts, 8)
    np.testing.assert_array_equal(eager, traced)
    streamed = np.stack(list(Batch32Generator(model, batch_size=32, max_seq_len=32).generate_streaming(prompts, 8)),
                        axis=1)
    np.testing.assert_array_equal(streamed, traced)


def test_full_width_two_layer_step_matches_oracle(cuda):
    """2B-4T widths (hidden 2560, FFN 6912, 20/5 heads, vocab 128256), 2 layers, batch 32."""
    from bitnet_tt.config import BitNet2B4TConfig
    from bitnet_tt.inference import Batch32Generator

    cfg = BitNet2B4TConfig(num_layers=2, max_position_embeddings=64)
    sd = _numpy_sd(cfg, seed=2026)
    model = _device_model(cfg, sd, cuda)
    prompts = np.random.default_rng(0).integers(0, cfg.vocab_size, size=(32, 2))
    gen = Batch32Generator(model, batch_size=32, max_seq_len=16, keep_logits=True)
    gen.prefill(prompts)
    dev_logits = gen.state.logits.float().cpu()
    oracle = om.OracleBitNet(cfg, sd, max_len=16)
    ref_tokens, ref_logits = oracle.generate(prompts, 1)
    rel = (dev_logits - ref_logits[0]).norm() / ref_logits[0].norm()
    assert rel < 2e-2, f"logits rel err {rel:.3e}"
    dev_tok = gen.state.ids.cpu().numpy()
    mismatch = dev_tok != ref_tokens[:, 0]
    assert not np.any(mismatch & ~_near_tie(ref_logits[0]).numpy())


@pytest.mark.parametrize("batch,full", [(32, False), (4, False), (32, True)])
def test_persistent_decode_equals_per_op_path(cuda, batch, full):
    """The all-layer persistent launch against the per-operation launches:
    ids, hidden states, logits and KV caches bit-identical, including ragged
    contexts past one attention split (256 keys)."""
    from bitnet_tt import _lib
    from bitnet_tt.config import BitNet2B4TConfig
    from bitnet_tt.inference import Batch32Generator

    cfg = BitNet2B4TConfig(num_layers=2, max_position_embeddings=512) if full else _small_cfg()
    sd = _numpy_sd(cfg, seed=11)
    model = _device_model(cfg, sd, cuda)
    rng = np.random.default_rng(batch + full)
    prompts = rng.integers(0, cfg.vocab_size, size=(batch, 3))
    gens = [Batch32Generator(model, batch_size=batch, max_seq_len=640, keep_logits=True, persistent=p)
            for p in (True, False)]
    assert gens[0].persistent and not gens[1].persistent
    pos = torch.from_numpy(rng.integers(100, 600, size=batch).astype(np.int32))
    for g in gens:
        g.set_context_limit(640)
        g.prefill(prompts)
        g.state.positions.copy_(pos)  # jump ahead: rows up to 599, up to three attention splits
    for _ in range(3):
        for g in gens:
            g.step()
        a, b = gens[0].state, gens[1].state
        assert torch.equal(a.hidden, b.hidden)
        assert torch.equal(a.logits, b.logits)
        assert torch.equal(a.ids, b.ids)
        assert torch.equal(a.positions, b.positions)
    for ca, cb in zip(gens[0].state.caches, gens[1].state.caches):
        assert torch.equal(ca.key_cache, cb.key_cache)
        assert torch.equal(ca.value_cache, cb.value_cache)
    assert _lib.last_device_status()[0] == 0


@pytest.mark.parametrize("b,nshard", [(32, 3), (64, 8), (4, 2)])
def test_vocab_sharded_lm_head_equals_unsharded(cuda, b, nshard):
    """Shard kernels + pair merge (what each rank of a vocabulary-split run
    does) against the single-table lm_head + argmax: identical ids."""
    from bitnet_tt import _lib
    from bitnet_tt.inference.vocab_shard import shard_bounds

    v, k = 1000, 512
    g = torch.Generator().manual_seed(b * 7 + nshard)
    h = torch.randn((b, k), generator=g).to(torch.bfloat16).to(cuda)
    e = (0.05 * torch.randn((v, k), generator=g)).to(torch.bfloat16)
    e[777] = e[5]  # an exact tie across shards: the smaller index must win
    h[1] = 0       # a row where every logit ties
    tiled = _lib.pack_lm_head(e.to(cuda))
    ws = torch.zeros(_lib.argmax_workspace_bytes(b, k, v), dtype=torch.uint8, device=cuda)
    ref = torch.empty(b, dtype=torch.int32, device=cuda)
    _lib.lm_head_argmax(h, tiled, v, ws, ref)
    pairs = torch.zeros((nshard, b, 2), dtype=torch.float32, device=cuda)
    tile_bytes = (k // 8) * 2048
    for r in range(nshard):
        t0, t1, r0, rows = shard_bounds(v, nshard, r)
        wsr = torch.zeros(_lib.argmax_workspace_bytes(b, k, max(rows, 1)), dtype=torch.uint8, device=cuda)
        _lib.lm_head_argmax_shard(h, tiled[t0 * tile_bytes:t1 * tile_bytes], rows, r0, wsr, pairs[r])
    ids = torch.empty(b, dtype=torch.int32, device=cuda)
    pos = torch.zeros(b, dtype=torch.int32, device=cuda)
    _lib.argmax_merge_pairs(pairs, ids, pos)
    torch.cuda.synchronize()
    assert _lib.last_device_status()[0] == 0
    assert torch.equal(ids, ref)
    assert int(ids[1]) == 0
    assert torch.equal(pos.cpu(), torch.ones(b, dtype=torch.int32))


def test_checkpoint_and_packed_cache_load_identically(cuda, tmp_path):
    """HF-layout safetensors -> load_bitnet_weights -> device packing gives the
    same device tensors as loading the (bf16-rounded) state dict directly; the
    packed cache (save_packed_weights / load_packed_weights) reproduces them
    byte for byte without packing, and a model from it decodes the same ids."""
    from bitnet_tt.inference import Batch32Generator
    from bitnet_tt.model import create_model
    from bitnet_tt.utils.weights import (load_bitnet_weights, load_packed_weights, save_hf_checkpoint,
                                         save_packed_weights)

    cfg = _small_cfg()
    sd = {k: torch.from_numpy(v).to(torch.bfloat16).float().numpy() for k, v in _numpy_sd(cfg, seed=19).items()}
    save_hf_checkpoint(sd, cfg, str(tmp_path / "ckpt"), max_shard_bytes=1 << 20)
    sd2, cfg2 = load_bitnet_weights(str(tmp_path / "ckpt"))
    direct = _device_model(cfg, sd, cuda)
    from_ckpt = _device_model(cfg2, sd2, cuda)
    save_packed_weights(from_ckpt, str(tmp_path / "packed.safetensors"))
    cached = create_model(cfg2, cuda)
    load_packed_weights(cached, str(tmp_path / "packed.safetensors"))

    def tensors(m):
        out = [m.embed_tokens.weight_tiled, m.lm_head_tiled, m.norm.weight]
        for layer in m.layers:
            a, f = layer.self_attn, layer.mlp
            out += [a.qkv_proj.weight, a.o_proj.weight, f.gate_up_proj.weight, f.down_proj.weight,
                    layer.input_layernorm.weight, layer.post_attention_layernorm.weight, a.attn_sub_norm.weight,
                    f.ffn_sub_norm.weight]
        return out

    for m in (from_ckpt, cached):
        for x, y in zip(tensors(direct), tensors(m)):
            assert torch.equal(x, y)
        for la, lb in zip(direct.layers, m.layers):
            for pa, pb in ((la.self_attn.qkv_proj, lb.self_attn.qkv_proj), (la.mlp.gate_up_proj, lb.mlp.gate_up_proj),
                           (la.mlp.down_proj, lb.mlp.down_proj)):
                assert pa.segments().count == pb.segments().count
                assert list(pa.segments().scale) == list(pb.segments().scale)
    assert cached.lm_head_tiled is cached.embed_tokens.weight_tiled  # tied head stays one table
    prompts = np.random.default_rng(4).integers(0, cfg.vocab_size, size=(4, 5))
    ids = [Batch32Generator(m, batch_size=4, max_seq_len=32).generate(prompts, 4) for m in (direct, cached)]
    np.testing.assert_array_equal(ids[0], ids[1])
    other = create_model(_small_cfg(hidden_size=384, num_attention_heads=3, num_key_value_heads=1), cuda)
    with pytest.raises(ValueError):
        load_packed_weights(other, str(tmp_path / "packed.safetensors"))
