"""bitnet_bitlinear_noalloc: the BitLinear entry point for callers that cannot
allocate device memory where they call (an FFI host without a CUDA allocator,
code that must not allocate).  Its quantised activations live in a static
device array of the library instead of caller buffers.

The test calls it through the C ABI and compares it with the allocating entry
point bitnet_bitlinear (caller-owned buffers) on two calls in a row with
different inputs; results must be bit-exact, as for every BitLinear test.
The file sorts last so that a run stopping at its first failure has already
run every other test."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_both(cuda, m, k, n, epilogue, seed, path):
    from bitnet_tt import _lib

    lib = _lib.load()
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g).to(torch.bfloat16).to(cuda)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).to(cuda)
    w = torch.from_numpy(np.random.default_rng(seed).integers(-1, 2, size=(n, k)).astype(np.int8)).to(cuda)
    wp = _lib.pack_ternary(w)
    if epilogue == _lib.EPI_RELU2_MUL:
        seg, n_out = _lib.Segments.make([n // 2, n], [0.02, 0.03]), n // 2
    else:
        seg, n_out = _lib.Segments.make([n], [0.025]), n
    res = torch.randn((m, n), generator=g).to(torch.bfloat16).to(cuda) if epilogue == _lib.EPI_RESIDUAL_ADD else None
    bufs = _lib.ActBuffers(m, k, cuda)
    y_ref = torch.empty((m, n_out), dtype=torch.bfloat16, device=cuda)
    acc_ref = torch.empty((m, n), dtype=torch.int32, device=cuda)
    y_new = torch.empty_like(y_ref)
    acc_new = torch.empty_like(acc_ref)
    s = _lib.stream_handle()
    st = lib.bitnet_bitlinear(_lib.ptr(x), m, k, _lib.ptr(gamma), 1e-5, _lib.ptr(wp), n, ctypes.byref(seg), epilogue,
                              _lib.ptr(res), _lib.ptr(y_ref), _lib.ptr(acc_ref), _lib.ptr(bufs.q),
                              _lib.ptr(bufs.row_scale), _lib.ptr(bufs.row_sum), path, s)
    assert st == 0, _lib.status_string(st)
    st = lib.bitnet_bitlinear_noalloc(_lib.ptr(x), m, k, _lib.ptr(gamma), 1e-5, _lib.ptr(wp), n, ctypes.byref(seg),
                                      epilogue, _lib.ptr(res), _lib.ptr(y_new), _lib.ptr(acc_new), path, s)
    assert st == 0, _lib.status_string(st)
    torch.cuda.synchronize()
    assert _lib.last_device_status()[0] == 0
    return y_ref, acc_ref, y_new, acc_new


@pytest.mark.parametrize("m,k,n,epi,path", [
    (32, 2560, 3840, 0, 2),   # decode QKV shape, tcgen05 path
    (32, 6912, 2560, 2, 2),   # decode down shape with the residual epilogue
    (1, 2560, 13824, 1, 1),   # batch-1 gate/up, ReLU^2 epilogue: the fused SIMT launch (uses no scratch)
    (3, 2500, 2560, 2, 1),    # SIMT path through the static scratch: K % 8 != 0 takes the act-quant
                              # launch into the scratch, then the CUDA-core BitLinear reads it
])
def test_noalloc_matches_allocating_entry_point_twice(cuda, m, k, n, epi, path):
    for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
        y_ref, acc_ref, y_new, acc_new = _call_both(cuda, m, k, n, epi, seed + 100 * m, path)
        np.testing.assert_array_equal(acc_new.cpu().numpy(), acc_ref.cpu().numpy(), err_msg=f"call {call}")
        np.testing.assert_array_equal(y_new.view(torch.int16).cpu().numpy(), y_ref.view(torch.int16).cpu().numpy(),
                                      err_msg=f"call {call}")


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    from bitnet_tt import _lib

    lib = _lib.load()
    y = torch.empty((512, 128), dtype=torch.bfloat16, device=cuda)
    x = torch.zeros((512, 4096), dtype=torch.bfloat16, device=cuda)
    wp = torch.zeros(_lib.packed_weight_bytes(128, 4096), dtype=torch.uint8, device=cuda)
    # 512 token rows > 256, and 512 x 4096 bytes > 1 MiB
    st = lib.bitnet_bitlinear_noalloc(_lib.ptr(x), 512, 4096, None, 1e-5, _lib.ptr(wp), 128, None, 0, None,
                                      _lib.ptr(y), None, 0, _lib.stream_handle())
    assert st == -6
    assert "static scratch" in _lib.status_string(st)
    # 256 rows x 8192 K = 2 MiB > 1 MiB
    st = lib.bitnet_bitlinear_noalloc(_lib.ptr(x), 256, 8192, None, 1e-5, _lib.ptr(wp), 128, None, 0, None,
                                      _lib.ptr(y), None, 0, _lib.stream_handle())
    assert st == -6
