"""BitLinear and RMSNorm layers on the B200 kernels.

Mirrors the reference's src/bitnet_tt/layers/bitlinear.py:
  * Linear(in_features, out_features, device, compute_fidelity, weight_dtype)
    with load_weights (W [out, in]), load_pretransposed_weight (W^T [in, out]
    already ternary, plus its scale), __call__(x, norm_weight, norm_epsilon)
    and the weight_scale / _use_packed_ternary / weight attributes
    (reference bitlinear.py:132-353);
  * RMSNorm(hidden_size, device, eps) with load_weights / __call__
    (reference bitlinear.py:356-461).
Only the packed_ternary weight dtype exists here: the weights live in the 2-bit
device layout and __call__ runs the fused RMSNorm + int8 quant + ternary
contraction + scale kernels (bitnet_act_quant + bitnet_bitlinear_q).
"""

from __future__ import annotations

import threading

import numpy as np
import torch

from .. import _lib
from ..utils.quantization import weight_quant_ternary

_WS_LOCK = threading.Lock()
_WORKSPACES: dict[tuple, _lib.ActBuffers] = {}


def _workspace(m: int, k: int, device: torch.device) -> _lib.ActBuffers:
    """Activation buffers shared by eager Linear calls (keyed by shape and device)."""
    key = (device.index, m, k)
    with _WS_LOCK:
        ws = _WORKSPACES.get(key)
        if ws is None:
            ws = _lib.ActBuffers(m, k, device)
            _WORKSPACES[key] = ws
    return ws


def quantize_ternary(weight) -> tuple[torch.Tensor, float]:
    """W [out, in] -> (int8 ternary codes, absmean scale).

    NumPy input follows the reference quantiser bit for bit (host, load time);
    torch input is quantised with the same formula where it lives (used for
    synthetic weights generated on the GPU)."""
    if isinstance(weight, np.ndarray):
        q, s = weight_quant_ternary(weight.astype(np.float32))
        return torch.from_numpy(q), float(s)
    w = weight.float()
    s = torch.clamp(w.abs().mean(), min=1e-5)
    q = torch.clamp(torch.round(w / s), -1, 1).to(torch.int8)
    return q, float(s)


def quantize_and_transpose_weight(weight: np.ndarray) -> tuple[np.ndarray, float]:
    """Reference bitlinear.py:104-114: ternary W^T [in, out] (float32) and the scale."""
    q, s = weight_quant_ternary(weight.astype(np.float32))
    return q.T.astype(np.float32).copy(), float(s)


def _as_device(t, device: torch.device, dtype: torch.dtype | None = None) -> torch.Tensor:
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device).contiguous()


class Linear:
    """Packed-ternary BitLinear.  y = bf16(acc * weight_scale / s_token)."""

    def __init__(self, in_features: int, out_features: int, device=None, compute_fidelity: str = "hifi2",
                 weight_dtype: str = "packed_ternary") -> None:
        if weight_dtype != "packed_ternary":
            raise ValueError(
                f"weight_dtype={weight_dtype!r}: the B200 build implements the packed_ternary path only"
            )
        self.in_features = in_features
        self.out_features = out_features
        self.device = torch.device(device if device is not None else "cuda")
        self.weight: torch.Tensor | None = None  # device weight layout (uint8)
        self.weight_scale: float = 1.0
        self._fidelity = compute_fidelity
        self._weight_dtype_name = weight_dtype
        self._use_packed_ternary = True
        self._segments: list[tuple[int, float]] | None = None
        self.epilogue = _lib.EPI_NONE

    # ---- loading ----------------------------------------------------------
    def load_ternary(self, w_q, scale: float = 1.0, segments: list[tuple[int, float]] | None = None) -> None:
        """Load int8 ternary codes W_q [out, in] with a scale (or per-row-range scales)."""
        w_q = _as_device(w_q, self.device, torch.int8)
        if tuple(w_q.shape) != (self.out_features, self.in_features):
            raise ValueError(f"weight shape {tuple(w_q.shape)} != ({self.out_features}, {self.in_features})")
        self.weight = _lib.pack_ternary(w_q)
        self.weight_scale = float(scale)
        self._segments = segments
        self._use_packed_ternary = True

    def load_weights(self, weight) -> None:
        """Quantise W [out, in] (absmean ternary) and pack it (reference bitlinear.py:199-254)."""
        q, s = quantize_ternary(weight)
        self.load_ternary(q, s)

    def load_pretransposed_weight(self, weight_t, scale: float = 1.0) -> None:
        """Load an already-ternary W^T [in, out] with its post-matmul scale
        (reference bitlinear.py:256-307)."""
        wt = weight_t if isinstance(weight_t, torch.Tensor) else torch.from_numpy(np.asarray(weight_t))
        self.load_ternary(torch.round(wt.float()).clamp(-1, 1).to(torch.int8).t().contiguous(), scale)

    def load_tilized(self, tiles, scale: float = 1.0) -> None:
        """Load a ternary weight already in the reference's Tensix tile format
        (uint8 [tiles, 256] from kernels/pack.py pack_ternary_tilized of W [out, in],
        the tiling the packed_ternary load_weights stores, bitlinear.py:211-251),
        re-laid out on the device without unpacking on the host."""
        t = _as_device(tiles, self.device, torch.uint8).reshape(-1)
        self.weight = _lib.pack_from_tilized(t, self.out_features, self.in_features)
        self.weight_scale = float(scale)
        self._segments = None
        self._use_packed_ternary = True

    def set_segments(self, segments: list[tuple[int, float]] | None) -> None:
        """Per-row-range scales of a fused projection: [(end_row, scale), ...]."""
        self._segments = segments

    def segments(self) -> _lib.Segments:
        if self._segments:
            return _lib.Segments.make([e for e, _ in self._segments], [s for _, s in self._segments])
        return _lib.Segments.make([self.out_features], [self.weight_scale])

    @property
    def output_features(self) -> int:
        return self.out_features // 2 if self.epilogue == _lib.EPI_RELU2_MUL else self.out_features

    # ---- forward ----------------------------------------------------------
    def forward_into(self, bufs: _lib.ActBuffers, m: int, y: torch.Tensor, residual: torch.Tensor | None = None,
                     acc_out: torch.Tensor | None = None, path: int = _lib.PATH_AUTO) -> None:
        """Run the ternary contraction on already-quantised activations in `bufs`."""
        epi = self.epilogue if residual is None else _lib.EPI_RESIDUAL_ADD
        _lib.bitlinear_q(bufs, m, self.in_features, self.weight, self.out_features, self.segments(), epi,
                         residual, y, acc_out=acc_out, path=path)

    def forward_fused(self, x: torch.Tensor, norm_weight: torch.Tensor | None, eps: float, bufs: _lib.ActBuffers,
                      y: torch.Tensor, residual: torch.Tensor | None = None) -> None:
        """Norm + act-quant + contraction from bf16 rows x [M, in] (bitnet_bitlinear:
        one launch below the ridge batch, two above; `bufs` holds the codes)."""
        epi = self.epilogue if residual is None else _lib.EPI_RESIDUAL_ADD
        _lib.bitlinear_fused(x, norm_weight, eps, bufs, self.weight, self.out_features, self.segments(), epi,
                             residual, y)

    def __call__(self, x: torch.Tensor, norm_weight: torch.Tensor | None = None,
                 norm_epsilon: float | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("Weights not loaded. Call load_weights() first.")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"input features {x.shape[-1]} != {self.in_features}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).to(torch.bfloat16).contiguous()
        m = x2.shape[0]
        ws = _workspace(m, self.in_features, x2.device)
        gamma = norm_weight.reshape(-1).to(torch.bfloat16).contiguous() if norm_weight is not None else None
        eps = 1e-5 if norm_epsilon is None else float(norm_epsilon)
        _lib.act_quant(x2, gamma, eps, ws)
        y = torch.empty((m, self.output_features), dtype=torch.bfloat16, device=x2.device)
        res = residual.reshape(m, -1).contiguous() if residual is not None else None
        self.forward_into(ws, m, y, residual=res)
        return y.reshape(*lead, self.output_features)


class RMSNorm:
    """RMSNorm in bf16 (HF BitNetRMSNorm semantics) on the act-quant kernel."""

    def __init__(self, hidden_size: int, device=None, eps: float = 1e-6) -> None:
        self.hidden_size = hidden_size
        self.device = torch.device(device if device is not None else "cuda")
        self.eps = eps
        self.weight: torch.Tensor | None = None

    def load_weights(self, weight) -> None:
        self.weight = _as_device(np.asarray(weight, dtype=np.float32).reshape(-1) if isinstance(weight, np.ndarray)
                                 else weight.reshape(-1), self.device, torch.bfloat16)

    def enable_sharded_fast_path(self, num_cores: int = 8) -> bool:
        """The reference's Tensix core-grid option (bitlinear.py:406-431); a no-op here."""
        return True

    def __call__(self, x: torch.Tensor, memory_config=None) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("RMSNorm weights not loaded")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        return _lib.rmsnorm(x2, self.weight, self.eps).reshape(*lead, self.hidden_size)
