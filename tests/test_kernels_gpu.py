"""GPU parity of the packing, quantisation and BitLinear kernels against the
CPU oracle, through the C ABI.  Integer results (packed bytes, int8 codes,
row sums, int32 accumulators) must be bit-exact; the bf16 outputs follow the
oracle's rounding points and must match bit for bit as well."""

import numpy as np
import pytest
import torch

from oracle import bitlinear as ob
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _lib():
    from bitnet_tt import _lib as L

    return L


def rand_bf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)


def rand_ternary(n, k, seed, p0=0.4):
    rng = np.random.default_rng(seed)
    return rng.choice(np.array([-1, 0, 1], np.int8), size=(n, k), p=[(1 - p0) / 2, p0, (1 - p0) / 2])


def f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


# ---------------------------------------------------------------------------
# packing
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n,k", [(128, 64), (130, 70), (3840, 2560), (64, 6912), (1, 1)])
def test_pack_ternary_bytes(cuda, n, k):
    L = _lib()
    w = rand_ternary(n, k, seed=n * 7 + k)
    dev = L.pack_ternary(torch.from_numpy(w).to(cuda))
    np.testing.assert_array_equal(dev.cpu().numpy(), ob.device_pack(w))


@pytest.mark.parametrize("n,k", [(128, 64), (5, 7), (256, 2560)])
def test_pack_from_canonical_bytes(cuda, n, k):
    L = _lib()
    w = rand_ternary(n, k, seed=k)
    canon = oq.pack_ternary_weights(w)
    dev = L.pack_from_canonical(torch.from_numpy(canon).to(cuda), n, k)
    np.testing.assert_array_equal(dev.cpu().numpy(), ob.device_pack(w))


@pytest.mark.parametrize("name,n,k", [("tl", 64, 128), ("tlo", 50, 100)])
def test_pack_from_tilized_golden_tiles(cuda, golden, name, n, k):
    """The reference's own tilized bytes (golden vectors made by its kernels/pack.py)
    re-laid out on the device equal the device packing of the same codes."""
    L = _lib()
    tiles = golden[f"{name}_packed"]
    w = golden[f"{name}_in"].astype(np.int8)
    assert tiles.size == L.tilized_weight_bytes(n, k)
    dev = L.pack_from_tilized(torch.from_numpy(np.ascontiguousarray(tiles)).to(cuda), n, k)
    np.testing.assert_array_equal(dev.cpu().numpy(), ob.device_pack(w))


@pytest.mark.parametrize("n,k", [(640, 2560), (2560, 6912), (33, 95)])
def test_pack_from_tilized_bytes(cuda, n, k):
    L = _lib()
    w = rand_ternary(n, k, seed=n + 3 * k)
    tiles, _ = oq.pack_ternary_tilized(w, 1.0)
    tiles[0, 0] |= 0b11  # a reserved code (last element of the first group) reads as a zero weight
    w_ref = w.copy()
    w_ref[3, 0] = 0  # tile element (k=0, n=3): face 0, index 3 -> bits 1..0 of byte 0
    dev = L.pack_from_tilized(torch.from_numpy(tiles).to(cuda), n, k)
    np.testing.assert_array_equal(dev.cpu().numpy(), ob.device_pack(w_ref))


def test_linear_load_tilized_matches_load_weights(cuda):
    from bitnet_tt.layers.bitlinear import Linear

    rng = np.random.default_rng(12)
    w = (0.02 * rng.standard_normal((384, 640))).astype(np.float32)
    wq, s = oq.weight_quant_ternary(w)
    tiles, _ = oq.pack_ternary_tilized(wq, float(s))
    a, b = Linear(640, 384, cuda), Linear(640, 384, cuda)
    a.load_weights(w)
    b.load_tilized(tiles, float(s))
    assert torch.equal(a.weight, b.weight) and a.weight_scale == b.weight_scale
    x = rand_bf16((8, 640), seed=4)
    assert torch.equal(a(x.to(cuda)), b(x.to(cuda)))


# ---------------------------------------------------------------------------
# fused RMSNorm + int8 absmax quantisation
# ---------------------------------------------------------------------------
def run_act_quant(x: torch.Tensor, gamma: torch.Tensor | None, eps: float, cuda):
    L = _lib()
    m, k = x.shape
    bufs = L.ActBuffers(m, k, cuda)
    normed = torch.empty((m, k), dtype=torch.bfloat16, device=cuda)
    L.act_quant(x.to(cuda), gamma.to(cuda) if gamma is not None else None, eps, bufs, normed_out=normed)
    torch.cuda.synchronize()
    q = ob.act_unlayout(bufs.q.cpu().numpy(), m, k)
    return q, f32(bufs.row_scale)[:m], bufs.row_sum.cpu().numpy()[:m], f32(normed)


@pytest.mark.parametrize("m,k", [(1, 64), (3, 100), (8, 2560), (32, 2560), (32, 6912), (40, 320), (300, 128),
                                 (2, 8192), (2, 8200),
                                 # many rows: one warp per row (prefill), both register budgets, ragged last tile
                                 (260, 2560), (520, 6912), (1024, 7168), (256, 8192),
                                 # the longest rows staged in shared memory, and the first that are not
                                 (264, 14336), (256, 14400)])
@pytest.mark.parametrize("with_gamma", [True, False])
def test_act_quant_bit_exact(cuda, m, k, with_gamma):
    x = rand_bf16((m, k), seed=m * 1000 + k)
    gamma = (1 + 0.1 * rand_bf16((k,), seed=k).float()).to(torch.bfloat16) if with_gamma else None
    q, s, rsum, normed = run_act_quant(x, gamma, 1e-5, cuda)
    ref = ob.bitlinear(f32(x), f32(gamma) if gamma is not None else None, 1e-5, np.zeros((1, k), np.int8))
    np.testing.assert_array_equal(normed, ref["normed"])
    np.testing.assert_array_equal(q, ref["q"])
    np.testing.assert_array_equal(s, ref["s"])
    np.testing.assert_array_equal(rsum, ref["row_sum"])


@pytest.mark.parametrize("reps", [1, 52])  # 5 rows (one CTA per row), 260 rows (one warp per row, prefill)
def test_act_quant_edge_rows(cuda, reps):
    k = 96
    x = np.zeros((5, k), np.float32)
    x[1, :] = 1e4 * np.linspace(-1, 1, k)        # large values
    x[2, 0] = 127.0                               # KAT: absmax 127 -> scale 1
    x[2, 1:8] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5]  # exact .5 ties
    x[3, :] = 1e-30                               # below the 1e-5 absmax clamp
    x[4, :] = np.linspace(-3, 3, k)
    xt = torch.from_numpy(np.tile(x, (reps, 1))).to(torch.bfloat16)
    q, s, rsum, _ = run_act_quant(xt, None, 1e-5, cuda)
    ref = ob.bitlinear(f32(xt), None, 1e-5, np.zeros((1, k), np.int8))
    np.testing.assert_array_equal(q, ref["q"])
    np.testing.assert_array_equal(s, ref["s"])
    np.testing.assert_array_equal(rsum, ref["row_sum"])
    for j in range(0, 5 * reps, 5):
        assert s[j + 2] == 1.0 and q[j + 2, :8].tolist() == [127, 0, 2, 2, 0, -2, -2, 4]
        assert not q[j].any() and not q[j + 3].any()


# ---------------------------------------------------------------------------
# BitLinear
# ---------------------------------------------------------------------------
def run_bitlinear(cuda, x, gamma, w_q, ends=None, scales=None, epilogue="none", residual=None, path=0,
                  eps=1e-5):
    L = _lib()
    m, k = x.shape
    n = w_q.shape[0]
    wp = L.pack_ternary(torch.from_numpy(w_q).to(cuda))
    bufs = L.ActBuffers(m, k, cuda)
    L.act_quant(x.to(cuda), gamma.to(cuda) if gamma is not None else None, eps, bufs)
    epi = {"none": L.EPI_NONE, "relu2_mul": L.EPI_RELU2_MUL, "residual_add": L.EPI_RESIDUAL_ADD}[epilogue]
    seg = L.Segments.make(ends or [n], scales or [1.0]) if epilogue != "relu2_mul" else L.Segments.make([n // 2, n], scales)
    n_out = n // 2 if epilogue == "relu2_mul" else n
    y = torch.empty((m, n_out), dtype=torch.bfloat16, device=cuda)
    res = residual.to(cuda) if residual is not None else None
    acc = torch.empty((m, n), dtype=torch.int32, device=cuda)
    L.bitlinear_q(bufs, m, k, wp, n, seg, epi, res, y, acc_out=acc, path=path)
    torch.cuda.synchronize()
    st, site = L.last_device_status()
    assert st == 0, f"device status {st} at site {site}"
    return acc.cpu().numpy(), f32(y)


def check_bitlinear(cuda, m, n, k, path, epilogue="none", seed=0, split=0):
    L = _lib()
    x = rand_bf16((m, k), seed=seed + 1)
    gamma = (1 + 0.1 * rand_bf16((k,), seed=seed + 2).float()).to(torch.bfloat16)
    w = rand_ternary(n, k, seed=seed + 3)
    residual = rand_bf16((m, n), seed=seed + 4) if epilogue == "residual_add" else None
    if epilogue == "relu2_mul":
        ends, scales = None, [0.021, 0.017]
    elif n >= 384 and n % 128 == 0:
        ends, scales = [n - 256, n - 128, n], [0.02, 0.03, 0.015]  # QKV-like segments
    else:
        ends, scales = [n], [0.02]
    L.set_tc_split(split)
    try:
        acc, y = run_bitlinear(cuda, x, gamma, w, ends, scales, epilogue, residual, path)
    finally:
        L.set_tc_split(0)
    ref = ob.bitlinear(f32(x), f32(gamma), 1e-5, w, ends, scales, epilogue,
                       f32(residual) if residual is not None else None)
    np.testing.assert_array_equal(acc, ref["acc"])
    np.testing.assert_array_equal(y, ref["y"])


@pytest.mark.parametrize("m", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("n,k", [(128, 256), (130, 320), (384, 2560)])
def test_bitlinear_simt(cuda, m, n, k):
    check_bitlinear(cuda, m, n, k, path=1, seed=m + n + k)


@pytest.mark.parametrize("m", [1, 8, 16, 17, 32, 64, 200, 300])
@pytest.mark.parametrize("n,k", [(128, 256), (130, 320), (384, 2560)])
def test_bitlinear_tcgen05(cuda, m, n, k):
    check_bitlinear(cuda, m, n, k, path=2, seed=m * 3 + n + k)


@pytest.mark.parametrize("split", [1, 2, 3, 4, 7, 8])
def test_bitlinear_tcgen05_k_split(cuda, split):
    check_bitlinear(cuda, 32, 256, 2560, path=2, seed=split, split=split)


@pytest.mark.parametrize("path", [1, 2])
@pytest.mark.parametrize("epilogue", ["relu2_mul", "residual_add"])
@pytest.mark.parametrize("m", [1, 4, 32])
def test_bitlinear_epilogues(cuda, path, epilogue, m):
    if path == 1 and m > 8:
        pytest.skip("SIMT path serves M <= 8")
    check_bitlinear(cuda, m, 256, 640, path=path, epilogue=epilogue, seed=m + path)


@pytest.mark.parametrize("m,n,k,epilogue,split", [
    (32, 3840, 2560, "none", 0),          # qkv shape, automatic split (more CTAs than SMs)
    (32, 13824, 2560, "relu2_mul", 2),    # gate_up shape, 216 CTAs: two per SM, 256 TMEM columns
    (32, 2560, 6912, "residual_add", 8),  # down shape, 160 CTAs
    (16, 2560, 2560, "residual_add", 8),  # token tile 16
    (64, 2560, 2560, "residual_add", 0),  # 64 tokens, automatic split: one CTA per SM (shared memory)
    (64, 13824, 2560, "relu2_mul", 0),
])
def test_bitlinear_tcgen05_decode_shapes(cuda, m, n, k, epilogue, split):
    check_bitlinear(cuda, m, n, k, path=2, epilogue=epilogue, seed=n + k, split=split)


@pytest.mark.parametrize("m,n,k,epilogue", [
    (1000, 3840, 2560, "none"),           # prefill token tiles of 256, ragged last tile
    (4096, 2560, 6912, "residual_add"),   # down shape over 16 token tiles
    (2048, 1024, 2560, "relu2_mul"),
    # K > 16384: float(acc) through the conversion instruction instead of the exact 1.5 * 2^23 trick
    (300, 256, 16448, "relu2_mul"),
    (300, 384, 16448, "residual_add"),
])
def test_bitlinear_tcgen05_prefill_shapes(cuda, m, n, k, epilogue):
    check_bitlinear(cuda, m, n, k, path=2, epilogue=epilogue, seed=m + n)


@pytest.mark.parametrize("path", [1, 2])
def test_bitlinear_config0_full_size(cuda, path):
    """x [32, 2560], W [6912, 2560] with P(0) = 0.4, scale 0.02."""
    m = 32 if path == 2 else 8
    check_bitlinear(cuda, m, 6912, 2560, path=path, seed=2026)


def test_bitlinear_rejects_bad_arguments(cuda):
    L = _lib()
    w = torch.zeros(L.packed_weight_bytes(128, 64), dtype=torch.uint8, device=cuda)
    bufs = L.ActBuffers(4, 64, cuda)
    y = torch.empty((4, 128), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="invalid argument"):
        L.bitlinear_q(bufs, 4, 64, w, 128, None, 7, None, y)  # unknown epilogue
    with pytest.raises(RuntimeError, match="invalid argument"):
        L.bitlinear_q(bufs, 4, 64, w, 128, None, L.EPI_RESIDUAL_ADD, None, y)  # residual missing
    with pytest.raises(RuntimeError, match="invalid argument"):
        L.bitlinear_q(bufs, 9, 64, w, 128, None, L.EPI_NONE, None, y, path=L.PATH_SIMT)  # SIMT serves M <= 8
    with pytest.raises(RuntimeError, match="invalid argument"):
        L.bitlinear_q(bufs, 4, 64, w, 128, L.Segments.make([100], [1.0]), L.EPI_NONE, None, y)  # seg end != N


@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("epilogue", ["none", "relu2_mul", "residual_add"])
@pytest.mark.parametrize("k", [2560, 6912])
def test_fused_bitlinear_small_m_equals_two_launches(cuda, m, epilogue, k):
    """bitnet_bitlinear below the ridge batch: one kernel that normalises and
    quantises the token rows itself, bit-identical to act-quant + BitLinear."""
    L = _lib()
    n = 1024
    x = rand_bf16((m, k), seed=m * 10 + k).to(cuda)
    gamma = (1 + 0.1 * rand_bf16((k,), seed=k + 1).float()).to(torch.bfloat16).to(cuda)
    w = rand_ternary(n, k, seed=n + k)
    wp = L.pack_ternary(torch.from_numpy(w).to(cuda))
    epi = {"none": L.EPI_NONE, "relu2_mul": L.EPI_RELU2_MUL, "residual_add": L.EPI_RESIDUAL_ADD}[epilogue]
    seg = L.Segments.make([n // 2, n], [0.021, 0.017]) if epilogue == "relu2_mul" else L.Segments.make([n], [0.02])
    nout = n // 2 if epilogue == "relu2_mul" else n
    res = rand_bf16((m, nout), seed=5).to(cuda) if epilogue == "residual_add" else None
    ref_bufs = L.ActBuffers(m, k, cuda)
    L.act_quant(x, gamma, 1e-5, ref_bufs)
    y_ref = torch.empty((m, nout), dtype=torch.bfloat16, device=cuda)
    acc_ref = torch.empty((m, n), dtype=torch.int32, device=cuda)
    L.bitlinear_q(ref_bufs, m, k, wp, n, seg, epi, res, y_ref, acc_out=acc_ref, path=L.PATH_SIMT)
    bufs = L.ActBuffers(m, k, cuda)
    for _ in range(2):
        y = torch.zeros_like(y_ref)
        acc = torch.zeros_like(acc_ref)
        L.bitlinear_fused(x, gamma, 1e-5, bufs, wp, n, seg, epi, res, y, acc_out=acc)
        torch.cuda.synchronize()
        assert L.last_device_status()[0] == 0
        assert torch.equal(acc, acc_ref)
        assert torch.equal(y, y_ref)


def test_bounded_wait_gives_up_with_a_status_and_the_context_stays_usable(cuda):
    """A kernel whose wait can never complete (nothing arrives on its barrier)
    ends the wait after its cycle limit, records BITNET_ERR_DEVICE_TIMEOUT (site
    900) and returns; the status is read and cleared on the host, and the next
    kernels run normally."""
    L = _lib()
    assert L.last_device_status() == (0, 0)
    L.check(L.load().bitnet_selftest_bounded_wait(2_000_000, L.stream_handle()), "bitnet_selftest_bounded_wait")
    assert L.last_device_status() == (-5, 900)
    assert L.last_device_status() == (0, 0)  # read and cleared
    x = rand_bf16((8, 256), seed=9)
    q, s, rsum, _ = run_act_quant(x, None, 1e-5, cuda)
    ref = ob.bitlinear(f32(x), None, 1e-5, np.zeros((1, 256), np.int8))
    np.testing.assert_array_equal(q, ref["q"])
    assert L.last_device_status() == (0, 0)


@pytest.mark.filterwarnings("ignore:overflow encountered")
@pytest.mark.parametrize("k", [2560, 6912])
@pytest.mark.parametrize("reps", [1, 33])  # 8 rows (one CTA per row), 264 rows (one warp per row, prefill)
def test_act_quant_extreme_dynamic_range_rows(cuda, k, reps):
    """Rows at the edges of the bf16 range (1e-20 mixed with 1e17, magnitudes over
    2^-30 .. 2^30, an overflowing variance, subnormals only, ...): the kernel's
    codes, scales, row sums and normalised values equal the oracle's wherever the
    fp32 variance does not depend on the order of the fp64 sum of squares (every
    row here; a row whose variance did would be reported, not asserted)."""
    from extreme_rows import ROW_NAMES, extreme_rows, var_orders

    rows = extreme_rows(k, seed=k)
    gamma = (1 + 0.1 * rand_bf16((k,), seed=k + 1).float()).to(torch.bfloat16)
    x = torch.from_numpy(np.tile(rows, (reps, 1))).to(torch.bfloat16)
    q, s, rsum, normed = run_act_quant(x, gamma, 1e-5, cuda)
    ref = ob.bitlinear(rows, f32(gamma), 1e-5, np.zeros((1, k), np.int8))
    order_dependent = []
    for i, name in enumerate(ROW_NAMES):
        if len(set(var_orders(rows[i]).values())) != 1:
            order_dependent.append(name)
            continue
        for j in range(i, len(ROW_NAMES) * reps, len(ROW_NAMES)):
            np.testing.assert_array_equal(normed[j], ref["normed"][i], err_msg=name)
            np.testing.assert_array_equal(q[j], ref["q"][i], err_msg=name)
            assert s[j] == ref["s"][i] and rsum[j] == ref["row_sum"][i], name
    assert not order_dependent, f"rows whose fp32 variance depends on the summation order: {order_dependent}"
