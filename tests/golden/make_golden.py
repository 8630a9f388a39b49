"""Generate the golden fixtures that pin the oracle to the reference's own code.

Run in the build container, where the reference checkout is mounted:

    python tests/golden/make_golden.py /path/to/bitnet-tt

It imports the reference's pure-NumPy modules by file path
(src/bitnet_tt/utils/quantization.py and src/bitnet_tt/kernels/pack.py; the
rest of the package needs ttnn and cannot be imported), runs them on seeded
inputs and edge cases, and writes the inputs and outputs to
tests/golden/reference_quant.npz.  The GPU box never runs this script; the
tests read only the committed .npz.
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: str) -> None:
    quant = _load(os.path.join(ref_root, "src/bitnet_tt/utils/quantization.py"), "ref_quantization")
    pack = _load(os.path.join(ref_root, "src/bitnet_tt/kernels/pack.py"), "ref_pack")
    rng = np.random.default_rng(20260101)
    out: dict[str, np.ndarray] = {}

    # --- weight quantisation (quantization.py:15-57) ---
    w_cases = {
        "wq_rand": rng.standard_normal((64, 128)).astype(np.float32) * 0.02,
        "wq_large": rng.standard_normal((16, 40)).astype(np.float32) * 100.0,
        "wq_zero": np.zeros((8, 16), dtype=np.float32),
        # mean|W| = 1 exactly: W/s hits the .5 ties (half-to-even) and the clip
        "wq_ties": np.array([[0.5, -0.5, 1.5, -1.5, 0.5, -0.5, 1.5, -1.5],
                             [2.5, -2.5, 0.0, 0.0, 1.0, -1.0, 0.75, -0.25]], dtype=np.float32),
        "wq_odd": rng.standard_normal((7, 13)).astype(np.float32),
    }
    for name, w in w_cases.items():
        q, s = quant.weight_quant_ternary(w)
        out[f"{name}_in"] = w
        out[f"{name}_q"] = q
        out[f"{name}_s"] = np.asarray(s, dtype=np.float32)

    # --- activation quantisation (quantization.py:60-91) ---
    a_cases = {
        "aq_rand": rng.standard_normal((2, 16, 256)).astype(np.float32),
        "aq_rows": rng.standard_normal((32, 2560)).astype(np.float32),
        "aq_zero": np.zeros((3, 64), dtype=np.float32),
        "aq_kat127": np.concatenate([np.array([[127.0]], np.float32), np.zeros((1, 9), np.float32)], axis=1),
        # x * 127/amax lands exactly on k + 0.5 for amax = 127: ties to even
        "aq_ties": np.array([[127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5]], dtype=np.float32),
        "aq_large": (rng.standard_normal((4, 96)) * 1e4).astype(np.float32),
        "aq_tiny": (rng.standard_normal((4, 96)) * 1e-7).astype(np.float32),
    }
    for name, x in a_cases.items():
        q, s = quant.activation_quant_absmax(x)
        out[f"{name}_in"] = x
        out[f"{name}_q"] = q
        out[f"{name}_s"] = np.asarray(s, dtype=np.float32)

    # --- canonical 2-bit packing (quantization.py:111-174) ---
    p_cases = {
        "pk_rand": rng.integers(-1, 2, size=(48, 64)).astype(np.int8),
        "pk_odd": rng.integers(-1, 2, size=(5, 7)).astype(np.int8),   # flat padding crosses rows
        "pk_cfg0": rng.choice(np.array([-1, 0, 1], np.int8), size=(128, 256), p=[0.3, 0.4, 0.3]),
    }
    for name, w in p_cases.items():
        packed = quant.pack_ternary_weights(w)
        out[f"{name}_in"] = w
        out[f"{name}_packed"] = packed
        out[f"{name}_unpacked"] = quant.unpack_ternary_weights(packed, w.shape)

    # --- tilized Tensix packing (pack.py:101-203) ---
    wt = rng.standard_normal((64, 128)).astype(np.float32)
    wq, s = quant.weight_quant_ternary(wt)
    tp, ts = pack.pack_ternary_tilized(wq, float(s))
    out["tl_in"], out["tl_scale"] = wq, np.asarray(s, np.float32)
    out["tl_packed"], out["tl_scales"] = tp, ts
    out["tl_unpacked"] = pack.unpack_ternary_tilized(tp, ts, 128, 64)
    wo = rng.integers(-1, 2, size=(50, 100)).astype(np.int8)
    tpo, tso = pack.pack_ternary_tilized(wo, 0.5)
    out["tlo_in"], out["tlo_packed"] = wo, tpo
    out["tlo_unpacked"] = pack.unpack_ternary_tilized(tpo, tso, 100, 50)
    out["tl_bytes_2560x2560"] = np.asarray(pack.packed_dram_bytes(2560, 2560))
    out["tl_bytes_2560x6912"] = np.asarray(pack.packed_dram_bytes(2560, 6912))

    dst = os.path.join(HERE, "reference_quant.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst}: {len(out)} arrays, {os.path.getsize(dst)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python make_golden.py <path of a deveworld/bitnet-tt checkout>")
    main(sys.argv[1])
