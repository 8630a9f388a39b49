"""CPU oracle of the fused packed-ternary BitLinear and its device layouts.

The fused BitLinear of the B200 path is the reference's BitLinear call
(src/bitnet_tt/layers/bitlinear.py:309-353, fused RMSNorm of
src/bitnet_tt/inference/generator_batch32.py:718-727) with the activation
quantisation the reference defines in src/bitnet_tt/utils/quantization.py:60-91
(identical to HF ActQuant, transformers integrations/bitnet.py:244-249) and the
RMSNorm of HF BitNetRMSNorm (models/bitnet/modeling_bitnet.py:53-58) in bf16.
The rounding points are fixed as follows (the CUDA kernels follow them bit for
bit):

  ss   = sum x^2 in float64 (exact for bf16 inputs of sane dynamic range)
  var  = float32(ss / K);  r = 1 / sqrt(var + eps)         (float32, IEEE)
  a    = bf16(gamma * bf16(x * r))                        (no gamma: a = x)
  s    = 127 / max(max|a|, 1e-5);  q = clip(rint(a * s), -128, 127)
  acc  = sum_k q * W_q                                     (int32, exact)
  y    = bf16(float32(acc) * (w_scale / s))                (float32 divide, multiply)
  RELU2_MUL: h = bf16(bf16(relu(g)^2) * u) with g, u = y of the gate / up rows
  RESIDUAL_ADD: out = bf16(residual + y)
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def round_bf16(x) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(F32).reshape(x.shape)
    nan = np.isnan(x)
    return np.where(nan, x, out) if nan.any() else out


def bf16_bits(x) -> np.ndarray:
    """float32 values already on the bf16 grid -> uint16 bit patterns."""
    return (np.ascontiguousarray(round_bf16(x)).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(F32)


def rmsnorm_bf16(x: np.ndarray, gamma: np.ndarray | None, eps: float) -> np.ndarray:
    """RMSNorm of bf16 rows (x holds bf16 values as float32), bf16 result."""
    x = np.asarray(x, dtype=F32)
    if gamma is None:
        return x.copy()
    k = x.shape[-1]
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    var = (ss / float(k)).astype(F32)
    r = F32(1.0) / np.sqrt(var + F32(eps))
    y = round_bf16(x * r)
    return round_bf16(np.asarray(gamma, dtype=F32) * y)


def act_quant(a: np.ndarray):
    """quantization.py:60-91 on float32 rows -> (q int8, s float32[M], row_sum int32[M])."""
    a = np.asarray(a, dtype=F32)
    amax = np.maximum(np.max(np.abs(a), axis=-1), F32(1e-5)).astype(F32)
    s = (F32(127.0) / amax).astype(F32)
    q = np.clip(np.rint(a * s[:, None]), -128, 127).astype(np.int8)
    return q, s, q.astype(np.int64).sum(axis=-1).astype(np.int32)


def ternary_acc(q: np.ndarray, w_q: np.ndarray) -> np.ndarray:
    """acc[m, n] = sum_k q[m, k] * w_q[n, k], exact (float64 sums of small integers)."""
    return (q.astype(np.float64) @ w_q.astype(np.float64).T).astype(np.int64).astype(np.int32)


def scale_bf16(acc: np.ndarray, w_scale, s: np.ndarray) -> np.ndarray:
    """bf16(float32(acc) * (w_scale / s_m)); w_scale scalar or per-column array."""
    f = (np.asarray(w_scale, dtype=F32)[None, ...] / s[:, None]).astype(F32)
    return round_bf16(acc.astype(F32) * f)


def segment_scales(n: int, ends, scales) -> np.ndarray:
    col = np.empty(n, dtype=F32)
    start = 0
    for e, sc in zip(ends, scales):
        col[start:e] = sc
        start = e
    return col


def relu2_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    r = np.where(g > 0, round_bf16(g * g), F32(0.0)).astype(F32)
    return round_bf16(r * u)


def fused_gate_up_rows(f: int) -> tuple[np.ndarray, np.ndarray]:
    """Fused gate/up row order: 64-row groups [32 gate | 32 up].
    Returns (gate_rows, up_rows): fused row indices of gate[j] and up[j]."""
    j = np.arange(f)
    g = (j // 32) * 64 + (j % 32)
    return g, g + 32


def bitlinear(x: np.ndarray, gamma: np.ndarray | None, eps: float, w_q: np.ndarray, ends=None, scales=None,
              epilogue: str = "none", residual: np.ndarray | None = None) -> dict:
    """Full fused BitLinear.  x: bf16 values as float32 [M, K]; w_q int8 [N, K]
    (fused row order for 'relu2_mul').  Returns q, s, row_sum, acc, y."""
    n = w_q.shape[0]
    a = rmsnorm_bf16(x, gamma, eps)
    q, s, rsum = act_quant(a)
    acc = ternary_acc(q, w_q)
    if epilogue == "relu2_mul":
        gr, ur = fused_gate_up_rows(n // 2)
        g = scale_bf16(acc[:, gr], scales[0], s)
        u = scale_bf16(acc[:, ur], scales[1], s)
        y = relu2_mul(g, u)
    else:
        col = segment_scales(n, ends or [n], scales or [1.0])
        y = scale_bf16(acc, col, s)
        if epilogue == "residual_add":
            y = round_bf16(np.asarray(residual, dtype=F32) + y)
    return {"normed": a, "q": q, "s": s, "row_sum": rsum, "acc": acc, "y": y}


# --------------------------------------------------------------------------
# device layouts (restated so the packing kernels are checked byte for byte)
# --------------------------------------------------------------------------
def _ceil(x: int, m: int) -> int:
    return -(-x // m) * m


def device_pack(w_q: np.ndarray) -> np.ndarray:
    """int8 ternary [N, K] -> bytes of the device weight layout
    [N/128][K/64][128 rows][4 words]; word wi covers K offsets 16*wi + e,
    e = 4*j + b stored at bits 8*b + 2*j, code = w + 1 (invalid values -> 1)."""
    n, k = w_q.shape
    npad, kp = _ceil(n, 128), _ceil(k, 64)
    codes = np.ones((npad, kp), dtype=np.uint32)
    v = w_q.astype(np.int32)
    c = np.where(v == 1, 2, np.where(v == -1, 0, 1)).astype(np.uint32)
    codes[:n, :k] = c
    c6 = codes.reshape(npad // 128, 128, kp // 64, 4, 4, 4)  # nb, r, kc, wi, j, b
    j = np.arange(4).reshape(4, 1)
    b = np.arange(4).reshape(1, 4)
    shifts = (8 * b + 2 * j).astype(np.uint32)
    words = np.sum(c6 << shifts, axis=(-2, -1), dtype=np.uint64).astype(np.uint32)  # nb, r, kc, wi
    words = words.transpose(0, 2, 1, 3)  # nb, kc, r, wi
    return np.ascontiguousarray(words).view(np.uint8).reshape(-1)


def lm_head_pack(w_bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns [V, K] -> [V/128][K/8][128 rows][8 bf16] (uint16)."""
    v, k = w_bits.shape
    vpad, kp = _ceil(v, 128), _ceil(k, 8)
    out = np.zeros((vpad, kp), dtype=np.uint16)
    out[:v, :k] = w_bits
    return np.ascontiguousarray(out.reshape(vpad // 128, 128, kp // 8, 8).transpose(0, 2, 1, 3)).reshape(-1)


def act_rows(m: int) -> int:
    return _ceil(m, 16) if m <= 256 else _ceil(m, 256)


def act_tile(m: int) -> int:
    return _ceil(m, 16) if m <= 256 else 256


def act_unlayout(buf: np.ndarray, m: int, k: int) -> np.ndarray:
    """Device activation buffer -> int8 [m, k] (token tiles of T rows, inside a
    tile [K/16][T/8][8 rows][16 bytes])."""
    rows, t, kp = act_rows(m), act_tile(m), _ceil(k, 64)
    b = np.asarray(buf, dtype=np.int8)[: rows * kp].reshape(rows // t, kp // 16, t // 8, 8, 16)
    full = b.transpose(0, 2, 3, 1, 4).reshape(rows, kp)
    return full[:m, :k]
