"""Pin the CPU oracle to the reference: golden vectors produced by the
reference's own quantization.py / pack.py, and the reference tests' KATs
(tests/test_ternary_kernel.py, tests/test_bitlinear.py, tests/test_model.py)."""

import numpy as np
import pytest

from oracle import bitlinear as ob
from oracle import quant as oq


@pytest.mark.parametrize("name", ["wq_rand", "wq_large", "wq_zero", "wq_ties", "wq_odd"])
def test_weight_quant_matches_reference(golden, name):
    q, s = oq.weight_quant_ternary(golden[f"{name}_in"])
    np.testing.assert_array_equal(q, golden[f"{name}_q"])
    assert np.float32(s) == golden[f"{name}_s"]


def test_weight_quant_ties_half_to_even(golden):
    q = golden["wq_ties_q"]
    # mean|W| = 1: 0.5 -> 0, -0.5 -> 0, 1.5 -> 2 -> clip 1, 2.5 -> 2 -> clip 1
    assert q[0].tolist() == [0, 0, 1, -1, 0, 0, 1, -1]


@pytest.mark.parametrize("name", ["aq_rand", "aq_rows", "aq_zero", "aq_kat127", "aq_ties", "aq_large", "aq_tiny"])
def test_act_quant_matches_reference(golden, name):
    x = golden[f"{name}_in"]
    q, s = oq.activation_quant_absmax(x)
    np.testing.assert_array_equal(q, golden[f"{name}_q"])
    np.testing.assert_array_equal(s.astype(np.float32), golden[f"{name}_s"])
    # the fused oracle's quantiser is the same function on 2-D rows
    x2 = x.reshape(-1, x.shape[-1])
    q2, s2, rsum = ob.act_quant(x2)
    np.testing.assert_array_equal(q2, golden[f"{name}_q"].reshape(q2.shape))
    np.testing.assert_array_equal(s2, golden[f"{name}_s"].reshape(-1))
    np.testing.assert_array_equal(rsum, q2.astype(np.int64).sum(-1))


def test_act_quant_kat_scale_one(golden):
    # reference tests/test_model.py:91-102: max 127 -> scale 1.0
    assert np.allclose(golden["aq_kat127_s"], 1.0)
    assert golden["aq_ties_q"][0].tolist() == [127, 0, 2, 2, 0, -2, -2, 4]


@pytest.mark.parametrize("name", ["pk_rand", "pk_odd", "pk_cfg0"])
def test_canonical_pack_matches_reference(golden, name):
    w = golden[f"{name}_in"]
    packed = oq.pack_ternary_weights(w)
    np.testing.assert_array_equal(packed, golden[f"{name}_packed"])
    np.testing.assert_array_equal(oq.unpack_ternary_weights(packed, w.shape), golden[f"{name}_unpacked"])
    np.testing.assert_array_equal(golden[f"{name}_unpacked"], w)


def test_tilized_pack_matches_reference(golden):
    packed, scales = oq.pack_ternary_tilized(golden["tl_in"], float(golden["tl_scale"]))
    np.testing.assert_array_equal(packed, golden["tl_packed"])
    np.testing.assert_array_equal(scales, golden["tl_scales"])
    np.testing.assert_array_equal(oq.unpack_ternary_tilized(packed, scales, 128, 64), golden["tl_unpacked"])
    p2, s2 = oq.pack_ternary_tilized(golden["tlo_in"], 0.5)
    np.testing.assert_array_equal(p2, golden["tlo_packed"])
    np.testing.assert_array_equal(oq.unpack_ternary_tilized(p2, s2, 100, 50), golden["tlo_unpacked"])
    assert oq.packed_dram_bytes(2560, 2560) == int(golden["tl_bytes_2560x2560"])
    assert oq.packed_dram_bytes(2560, 6912) == int(golden["tl_bytes_2560x6912"])


# ---- the reference tests' own known answers, restated ----
def test_kat_encoding():
    # tests/test_ternary_kernel.py:31-39
    assert oq.encode_ternary_tt(np.array([-1, 0, 1, 0], np.int8)).tolist() == [0b10, 0b00, 0b01, 0b00]
    assert oq.decode_ternary_tt(np.array([0b10, 0b00, 0b01, 0b00], np.uint8)).tolist() == [-1, 0, 1, 0]


def test_kat_single_byte():
    # tests/test_ternary_kernel.py:58-62: -1, +1, 0, -1 -> 0b10_01_00_10
    assert oq.pack_4_to_byte(np.array([0b10, 0b01, 0b00, 0b10], np.uint8))[0] == 0b10_01_00_10


def test_kat_face_order():
    # tests/test_ternary_kernel.py:84-95
    t = np.zeros((32, 32), np.int8)
    t[0, 0], t[0, 16], t[16, 0], t[16, 16] = 1, 2, 3, 4
    f = oq.tile_to_faces(t)
    assert (f[0], f[256], f[512], f[768]) == (1, 2, 3, 4)
    np.testing.assert_array_equal(oq.faces_to_tile(oq.tile_to_faces(np.arange(1024).reshape(32, 32))),
                                  np.arange(1024).reshape(32, 32))


def test_kat_tile_counts():
    # tests/test_ternary_kernel.py:156-170
    assert oq.packed_tile_count(2560, 2560) == 80 * 80
    assert oq.packed_tile_count(2560, 6912) == 80 * 216
    assert 2560 * 2560 * 2 / oq.packed_dram_bytes(2560, 2560) > 7.5


def test_kat_sign_preserved():
    # tests/test_model.py:79-89
    q, _ = oq.weight_quant_ternary(np.array([[1.0, -1.0], [0.1, -0.1]], np.float32))
    assert q[0, 0] == 1 and q[0, 1] == -1


def test_kat_act_range_and_reconstruction():
    # tests/test_bitlinear.py:70-97
    x = np.random.default_rng(3).standard_normal((2, 16, 256)).astype(np.float32)
    q, s = oq.activation_quant_absmax(x)
    assert q.min() >= -128 and q.max() <= 127 and s.shape == (2, 16, 1)
    err = np.max(np.abs(x - q.astype(np.float32) / s))
    assert err <= np.max(np.max(np.abs(x), axis=-1, keepdims=True) / 127.0) + 1e-5


# ---- oracle self-consistency for the fused BitLinear ----
def test_round_bf16_ties_to_even():
    # 1 + 2^-8 is halfway between bf16 1.0 and 1 + 2^-7 -> rounds to 1.0 (even)
    assert ob.round_bf16(np.float32(1.0 + 2 ** -8)) == np.float32(1.0)
    assert ob.round_bf16(np.float32(1.0 + 3 * 2 ** -8)) == np.float32(1.0 + 2 ** -6)


def test_fused_bitlinear_matches_float_reference():
    rng = np.random.default_rng(0)
    m, k, n = 4, 256, 64
    x = ob.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    g = ob.round_bf16((1 + 0.1 * rng.standard_normal(k)).astype(np.float32))
    w = rng.integers(-1, 2, size=(n, k)).astype(np.int8)
    r = ob.bitlinear(x, g, 1e-5, w, [n], [0.02])
    # the int32 accumulator is the exact integer product
    np.testing.assert_array_equal(r["acc"], (r["q"].astype(np.int64) @ w.astype(np.int64).T))
    # and y approximates the float BitLinear (x_q / s) @ (w * ws)
    ref = (r["q"].astype(np.float64) / r["s"][:, None]) @ (w.astype(np.float64).T * 0.02)
    np.testing.assert_allclose(r["y"], ref, rtol=1e-2, atol=1e-3)


def test_device_pack_layout_roundtrip():
    rng = np.random.default_rng(1)
    w = rng.integers(-1, 2, size=(130, 70)).astype(np.int8)
    b = ob.device_pack(w)
    assert b.size == 256 * 128 // 4  # Npad=256, Kp=128: 2 bits per weight
    words = b.view(np.uint32).reshape(2, 2, 128, 4)  # nb, kc, r, wi
    for n, k in [(0, 0), (5, 17), (129, 69), (77, 63), (128, 64)]:
        nb, r, kc, kk = n // 128, n % 128, k // 64, k % 64
        wi, e = kk // 16, kk % 16
        j, bb = e // 4, e % 4
        code = (int(words[nb, kc, r, wi]) >> (8 * bb + 2 * j)) & 3
        assert code - 1 == w[n, k]
    # padding decodes to zero weights (code 1)
    assert ((int(words[1, 1, 127, 3]) >> 0) & 3) == 1
