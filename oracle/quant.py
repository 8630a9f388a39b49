"""NumPy restatement of the reference quantisers and 2-bit packers (oracle).

Each function cites the reference code it restates
(deveworld/bitnet-tt, paths inside that project).
"""

from __future__ import annotations

import numpy as np


# --------------------------------------------------------------------------
# src/bitnet_tt/utils/quantization.py
# --------------------------------------------------------------------------
def compute_weight_scale(weight: np.ndarray, eps: float = 1e-5):
    """quantization.py:15-29 -- s = max(mean|W|, eps) (float32 math for float32 W)."""
    return np.maximum(np.mean(np.abs(weight)), eps)


def weight_quant_ternary(weight: np.ndarray, eps: float = 1e-5):
    """quantization.py:32-57 -- W_q = clip(rint(W / s), -1, 1) as int8, and s."""
    s = compute_weight_scale(weight, eps)
    q = np.clip(np.round(weight / s), -1, 1).astype(np.int8)
    return q, s


def activation_quant_absmax(x: np.ndarray, num_bits: int = 8, eps: float = 1e-5):
    """quantization.py:60-91 -- per row: s = 127 / max(max|x|, eps);
    q = clip(rint(x * s), -128, 127)."""
    qb = 2 ** (num_bits - 1) - 1
    amax = np.maximum(np.max(np.abs(x), axis=-1, keepdims=True), eps)
    s = qb / amax
    q = np.clip(np.round(x * s), -qb - 1, qb).astype(np.int8)
    return q, s


def dequantize_weight(weight_quant: np.ndarray, scale) -> np.ndarray:
    """quantization.py:94-108."""
    return weight_quant.astype(np.float32) * float(scale)


def pack_ternary_weights(weight_quant: np.ndarray) -> np.ndarray:
    """quantization.py:111-138 -- flatten, code = w + 1, pad with code 1 to a
    multiple of 4, four codes per byte MSB first."""
    codes = weight_quant.astype(np.int32).reshape(-1) + 1
    pad = (-codes.size) % 4
    if pad:
        codes = np.concatenate([codes, np.ones(pad, dtype=np.int32)])
    c = codes.reshape(-1, 4)
    return ((c[:, 0] << 6) | (c[:, 1] << 4) | (c[:, 2] << 2) | c[:, 3]).astype(np.uint8)


def unpack_ternary_weights(packed: np.ndarray, original_shape) -> np.ndarray:
    """quantization.py:141-174 -- inverse of pack_ternary_weights."""
    p = packed.astype(np.uint8)
    codes = np.stack([(p >> 6) & 3, (p >> 4) & 3, (p >> 2) & 3, p & 3], axis=-1).reshape(-1)
    vals = codes.astype(np.int8) - 1
    n = int(np.prod(original_shape))
    return vals[:n].reshape(original_shape)


# --------------------------------------------------------------------------
# src/bitnet_tt/kernels/pack.py (Tensix tilized format; kept for its KATs,
# which pin the reference's 2-bit encoding)
# --------------------------------------------------------------------------
TILE = 32
FACE = 16
TILE_ELEMENTS = TILE * TILE
PACKED_TILE_BYTES = TILE_ELEMENTS // 4
ENC_NEG, ENC_ZERO, ENC_POS = 0b10, 0b00, 0b01  # pack.py:32-34


def encode_ternary_tt(values: np.ndarray) -> np.ndarray:
    """pack.py:37-42."""
    out = np.full(values.shape, ENC_ZERO, dtype=np.uint8)
    out[values == 1] = ENC_POS
    out[values == -1] = ENC_NEG
    return out


def decode_ternary_tt(codes: np.ndarray) -> np.ndarray:
    """pack.py:45-50."""
    out = np.zeros(codes.shape, dtype=np.int8)
    out[codes == ENC_POS] = 1
    out[codes == ENC_NEG] = -1
    return out


def pack_4_to_byte(codes: np.ndarray) -> np.ndarray:
    """pack.py:53-63 (MSB first)."""
    c = codes.astype(np.uint8).reshape(-1, 4)
    return ((c[:, 0] << 6) | (c[:, 1] << 4) | (c[:, 2] << 2) | c[:, 3]).astype(np.uint8)


def unpack_byte_to_4(packed: np.ndarray) -> np.ndarray:
    """pack.py:66-76."""
    p = packed.astype(np.uint8)
    return np.stack([(p >> 6) & 3, (p >> 4) & 3, (p >> 2) & 3, p & 3], axis=-1).reshape(-1)


def tile_to_faces(tile: np.ndarray) -> np.ndarray:
    """pack.py:79-86 -- four row-major 16x16 faces: TL, TR, BL, BR."""
    return np.concatenate([tile[:FACE, :FACE].ravel(), tile[:FACE, FACE:].ravel(),
                           tile[FACE:, :FACE].ravel(), tile[FACE:, FACE:].ravel()])


def faces_to_tile(flat: np.ndarray) -> np.ndarray:
    """pack.py:89-98."""
    f = [flat[i * FACE * FACE:(i + 1) * FACE * FACE].reshape(FACE, FACE) for i in range(4)]
    return np.concatenate([np.concatenate([f[0], f[1]], axis=1), np.concatenate([f[2], f[3]], axis=1)], axis=0)


def packed_tile_count(in_features: int, out_features: int) -> int:
    """pack.py:194-198."""
    return (-(-in_features // TILE)) * (-(-out_features // TILE))


def packed_dram_bytes(in_features: int, out_features: int) -> int:
    """pack.py:201-203."""
    return packed_tile_count(in_features, out_features) * PACKED_TILE_BYTES


def pack_ternary_tilized(weight_quant: np.ndarray, scale: float):
    """pack.py:101-155 -- tiles of W^T in row-major tile order, face order inside."""
    wt = weight_quant.T
    rows = -(-wt.shape[0] // TILE) * TILE
    cols = -(-wt.shape[1] // TILE) * TILE
    padded = np.zeros((rows, cols), dtype=np.int8)
    padded[:wt.shape[0], :wt.shape[1]] = wt
    tiles = []
    for tr in range(rows // TILE):
        for tc in range(cols // TILE):
            t = padded[tr * TILE:(tr + 1) * TILE, tc * TILE:(tc + 1) * TILE]
            tiles.append(pack_4_to_byte(encode_ternary_tt(tile_to_faces(t))))
    packed = np.stack(tiles) if tiles else np.zeros((0, PACKED_TILE_BYTES), np.uint8)
    return packed, np.full(len(tiles), scale, dtype=np.float32)


def unpack_ternary_tilized(packed: np.ndarray, tile_scales: np.ndarray, in_features: int, out_features: int):
    """pack.py:158-191."""
    rows = -(-in_features // TILE) * TILE
    cols = -(-out_features // TILE) * TILE
    out = np.zeros((rows, cols), dtype=np.float32)
    i = 0
    for tr in range(rows // TILE):
        for tc in range(cols // TILE):
            vals = decode_ternary_tt(unpack_byte_to_4(packed[i]))
            out[tr * TILE:(tr + 1) * TILE, tc * TILE:(tc + 1) * TILE] = faces_to_tile(vals).astype(np.float32) * \
                tile_scales[i]
            i += 1
    return out[:in_features, :out_features]
