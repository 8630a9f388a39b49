"""The C-ABI library loads without a GPU and exports every entry point that
include/bitnet_b200.h declares.  Only pure host helpers are called here."""

import ctypes
import os
import re

import pytest

from conftest import ROOT


def header_functions() -> list[str]:
    src = open(os.path.join(ROOT, "include", "bitnet_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bitnet_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from bitnet_tt import _lib

    lib = _lib.load()
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding declares a signature for every exported entry point
    assert sorted(_lib.exported_symbols()) == names


def header_arity() -> dict[str, int]:
    """Number of parameters of every function the header declares."""
    src = open(os.path.join(ROOT, "include", "bitnet_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(bitnet_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_binding_arity_matches_header():
    """Each ctypes signature declares as many arguments as the C prototype."""
    from bitnet_tt import _lib

    arity = header_arity()
    assert sorted(arity) == header_functions()
    wrong = {n: (len(_lib._SIGNATURES[n][1]), k) for n, k in arity.items() if len(_lib._SIGNATURES[n][1]) != k}
    assert not wrong, f"binding vs header argument counts differ: {wrong}"


def test_status_strings_and_sizes():
    from bitnet_tt import _lib

    lib = _lib.load()
    assert lib.bitnet_abi_version() == 3
    assert _lib.tilized_weight_bytes(2560, 2560) == 80 * 80 * 256
    assert _lib.tilized_weight_bytes(50, 100) == 8 * 256  # K and N padded to 32
    assert _lib.status_string(0) == "ok"
    assert "invalid argument" in _lib.status_string(-1)
    assert "unknown" in _lib.status_string(-99)
    # 2 bits per weight, rows padded to 128 and K to 64
    assert _lib.packed_weight_bytes(6912, 2560) == 6912 * 2560 // 4
    assert _lib.packed_weight_bytes(130, 70) == 256 * 128 // 4
    assert _lib.act_rows(1) == 16 and _lib.act_rows(32) == 32 and _lib.act_rows(300) == 512
    assert _lib.act_bytes(32, 2560) == 32 * 2560
    assert _lib.lm_head_bytes(128256, 2560) == 128256 * 2560 * 2
    # per-CTA (max, idx) pairs for up to 160 CTAs, then the hidden states tiled (K x T bf16)
    assert _lib.argmax_workspace_bytes(32, 2560, 128256) == 160 * 32 * 8 + 2560 * 32 * 2
    assert lib.bitnet_packed_weight_bytes(0, 5) == 0
    # attention: units per (sequence, KV head) from the wave model (at most one
    # per 256 keys); with more than one, 256-byte aligned counters, then per
    # unit 2G + 128G floats
    assert _lib.gqa_decode_workspace_bytes(32, 20, 5, 256) == 0
    assert _lib.gqa_decode_workspace_bytes(32, 20, 5, 257) == 768 + 32 * 5 * 2 * (8 + 512) * 4
    assert _lib.gqa_decode_workspace_bytes(32, 20, 5, 4096) == 768 + 32 * 5 * 5 * (8 + 512) * 4
    assert _lib.gqa_decode_workspace_bytes(1, 20, 5, 4096) == 256 + 5 * 16 * (8 + 512) * 4
    assert _lib.gqa_decode_workspace_bytes(256, 20, 5, 4352) == 0  # 1280 units of 4352 keys: one split
    # the counts measured best at config-4 contexts per GPU: 32 and 64 sequences -> 5 and 4 units
    assert _lib.gqa_decode_workspace_bytes(32, 20, 5, 4352) == 768 + 32 * 5 * 5 * (8 + 512) * 4
    assert _lib.gqa_decode_workspace_bytes(64, 20, 5, 4352) == 1280 + 64 * 5 * 4 * (8 + 512) * 4
    assert _lib.gqa_decode_workspace_bytes(32, 20, 3, 4096) == 0  # heads not a multiple of KV heads


def test_option_validation_is_host_side():
    from bitnet_tt import _lib

    with pytest.raises(RuntimeError):
        _lib.set_tc_split(9)
    with pytest.raises(RuntimeError):
        _lib.set_simt_max_m(-1)
    _lib.set_tc_split(0)
    _lib.set_simt_max_m(4)


def test_library_is_sm100a_only():
    """The .so carries sm_100a machine code (checked by its ELF note, not by disassembly)."""
    from bitnet_tt import _lib

    data = open(_lib.LIB_PATH, "rb").read()
    assert b"sm_100a" in data
