"""Activation rows at the edges of the bf16 range, shared by the CPU check of the
sum-of-squares exactness condition and the GPU act-quant parity test.

The norm's sum of squares is accumulated in fp64.  A square of a bf16 value has
at most 16 significant bits, so the sum of K squares is exact in every order
when the largest square is at most 2^(37 - ceil(log2 K)) times the smallest
nonzero one; beyond that the fp64 sum may round differently per order, and
var = fp32(ss / K) can then differ in the rare case that ss / K sits next to an
fp32 rounding boundary."""

from __future__ import annotations

import math

import numpy as np

from oracle import bitlinear as ob

ROW_NAMES = [
    "1e-20 and 1e17 mixed",
    "magnitudes log-uniform over 2^-6 .. 2^6 (inside the exact span)",
    "magnitudes log-uniform over 2^-30 .. 2^30 (beyond it)",
    "one 1e15 among 1e-3 values",
    "near-max bf16 values (3e38) with ones: var overflows fp32",
    "bf16 subnormals only (1e-39): var underflows",
    "zeros and a single 1e-38",
    "standard normal",
]


def extreme_rows(k: int, seed: int) -> np.ndarray:
    """[8, k] float32 holding bf16 values, one row per ROW_NAMES entry."""
    rng = np.random.default_rng(seed)
    sign = lambda: np.where(rng.random(k) < 0.5, -1.0, 1.0)  # noqa: E731
    rows = np.zeros((8, k), np.float64)
    rows[0] = sign() * np.where(rng.random(k) < 0.5, 1e-20, 1e17) * (1 + rng.random(k))
    rows[1] = sign() * np.exp2(rng.uniform(-6, 6, k))
    rows[2] = sign() * np.exp2(rng.uniform(-30, 30, k))
    rows[3] = sign() * 1e-3 * (1 + rng.random(k))
    rows[3, k // 3] = 1e15
    rows[4] = 1.0
    rows[4, ::7] = 3e38 * sign()[::7]
    rows[5] = sign() * 1e-39 * (1 + rng.random(k))
    rows[6, k // 2] = 1e-38
    rows[7] = rng.standard_normal(k)
    return ob.round_bf16(rows.astype(np.float32))


def var_orders(row: np.ndarray) -> dict[str, np.float32]:
    """fp32(ss / K) with ss summed in fp64 in several orders (and exactly)."""
    sq = row.astype(np.float64) ** 2
    k = row.size
    seq = 0.0
    for v in sq:
        seq += v
    rev = 0.0
    for v in sq[::-1]:
        rev += v
    sums = {"pairwise": float(np.sum(sq)), "sequential": seq, "reversed": rev, "exact": math.fsum(sq.tolist())}
    with np.errstate(over="ignore"):
        return {name: np.float32(s / k) for name, s in sums.items()}


def span_is_exact(row: np.ndarray) -> bool:
    """The documented exactness condition for this row."""
    sq = row.astype(np.float64) ** 2
    nz = sq[sq > 0]
    if nz.size == 0:
        return True
    return nz.max() <= nz.min() * 2.0 ** (37 - math.ceil(math.log2(row.size)))
