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
  converts once where it used to round and then convert);
* in the tiled code layout a row's 8-code chunks are contiguous and 32 chunks
  apart by a constant 256 T bytes (the prefill act-quant's pointer step)."""

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


def test_code_layout_steps_by_256_tiles_per_32_chunks():
    """The prefill act-quant stores a row's 8-code chunk ch = lane + 32 i at a
    pointer that starts at the chunk `lane` and grows by 256 T bytes per step
    (act_quant_rows_kernel), as one 8-byte store.  Both hold in the device code
    layout that oracle.bitlinear.act_unlayout reads (token tiles of T rows,
    inside a tile [K/16][T/8][8 rows][16 bytes])."""
    from oracle import bitlinear as ob

    for m_rows, k in ((300, 2560), (512, 6912), (256, 128), (264, 14336)):
        rows, t, kp = ob.act_rows(m_rows), ob.act_tile(m_rows), -(-k // 64) * 64
        assert t == 256
        # byte offset of (row, k) in the buffer, by the same reshape as act_unlayout
        off = np.arange(rows * kp, dtype=np.int64).reshape(rows // t, kp // 16, t // 8, 8, 16)
        off = off.transpose(0, 2, 3, 1, 4).reshape(rows, kp)
        chunks = kp // 8
        for lane in range(min(32, chunks)):
            ch = np.arange(lane, chunks, 32)
            start = off[:, 8 * ch]                                        # [rows, steps]
            np.testing.assert_array_equal(start, off[:, [8 * lane]] + (ch - lane)[None, :] // 32 * 256 * t)
            for e in range(8):                                            # 8 codes, 8 contiguous bytes
                np.testing.assert_array_equal(off[:, 8 * ch + e], start + e)
