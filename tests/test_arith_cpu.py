"""Host checks of the exact-arithmetic shortcuts the CUDA kernels take instead of
conversion instructions (the kernels' own results are checked bit for bit on the
GPU; these pin the identities those comments state, over the whole range the
kernels use them on):

* float(acc) as the fp32 with bits 0x4B400000 + acc, minus 1.5 * 2^23, is exact
  for |acc| < 2^22 (`i2f_exact`, csrc/epilogue.cuh; the BitLinear epilogues use
  it for K <= 16384, where |acc| <= 127 K);
* the int8 code rint(v) (half to even) is the low byte of fp32(v + 1.5 * 2^23)
  (`aq_rint_small` / `aq_codes4`, csrc/act_quant.cuh);
* with s = fp32(127 / amax) and |a| <= amax, |fp32(a * s)| < 127.5, so the codes
  need no clamp (`aq_codes4`);
* rounding a bf16-exact fp32 value to bf16 again changes nothing (the epilogue
  converts once where it used to round and then convert)."""

import numpy as np

MAGIC = np.float32(12582912.0)  # 1.5 * 2^23


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 (finite inputs)."""
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def test_int_to_float_by_magic_bits_is_exact_below_2_pow_22():
    acc = np.arange(-(1 << 22) + 1, 1 << 22, dtype=np.int64)  # every value the trick may see
    bits = (acc + 0x4B400000).astype(np.uint32)
    f = bits.view(np.float32) - MAGIC  # one fp32 subtraction, as __fsub_rn
    assert f.dtype == np.float32
    np.testing.assert_array_equal(f.astype(np.float64), acc.astype(np.float64))


def test_codes_are_the_low_byte_of_the_magic_sum():
    rng = np.random.default_rng(1)
    v = np.concatenate([
        rng.uniform(-127.5, 127.5, 2_000_000).astype(np.float32),
        (np.arange(-255, 256) / 2).astype(np.float32),  # every .5 tie in range
        np.nextafter(np.float32(0.5), np.float32(0)) * np.array([1, -1], np.float32),
        np.array([0.0, -0.0, 126.5, -126.5, 127.0, -127.0], np.float32),
    ])
    s = v + MAGIC  # fp32 add, round to nearest even
    q = np.rint(v.astype(np.float64)).astype(np.int64)  # half to even, as np.round
    np.testing.assert_array_equal(s.view(np.uint32).astype(np.int64) - 0x4B400000, q)
    np.testing.assert_array_equal(s.view(np.uint32) & 0xFF, (q & 0xFF).astype(np.uint32))


def test_scaled_codes_never_need_a_clamp():
    """Worst case a = amax over every finite positive bf16 amax (>= the 1e-5
    floor), and a one ulp below it: |fp32(a * fp32(127 / amax))| < 127.5."""
    b = np.arange(0x0001, 0x7F80, dtype=np.uint32) << 16  # positive finite bf16 values
    amax = np.maximum(b.view(np.float32), np.float32(1e-5))
    s = np.float32(127.0) / amax
    for a in (amax, _bf16_round(amax * np.float32(0.99609375))):
        v = (a * s).astype(np.float32)
        assert float(np.abs(v).max()) < 127.5
        assert int(np.abs(np.rint(v)).max()) <= 127


def test_bf16_rounding_is_idempotent():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(1_000_000) * np.exp(rng.uniform(-20, 20, 1_000_000))).astype(np.float32)
    once = _bf16_round(x)
    np.testing.assert_array_equal(_bf16_round(once), once)
