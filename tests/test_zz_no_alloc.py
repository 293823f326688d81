"""The allocation-free global sum (vox_cuda_global_sum_noalloc), called through the C ABI.

It exists for callers that cannot allocate device memory (a real-time audio callback, where cudaMalloc can block and
synchronise the device; a plugin host that owns all device memory except the inputs and outputs it passes). Its
result must equal the allocating entry point's (vox_cuda_global_sum_partials + vox_cuda_global_sum_finish) on two
calls in a row: the second call reuses the library's scratch array left over from the first. This file is collected
last so that a run stopping at its first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

F32, BF16 = 0, 1


def _noalloc(vox):
    f = vox.lib.vox_cuda_global_sum_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _reference_path(vox, x):
    """The allocating entry points, caller scratch: partials for the whole tensor, then the fold."""
    rows, n = x.shape
    return vox.global_sum_finish(vox.global_sum_partials(x, 0, rows)).item()


@pytest.mark.parametrize("rows", [3000, 0, 1, 839, 841])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_global_sum_matches_the_allocating_entry_point(vox, port, dtype, rows):
    """Row counts below, at and above the 840 slots (most slots empty, one row per slot, a wrapped slot) and none."""
    f = _noalloc(vox)
    n = 4096
    x = torch.from_numpy(port.normal((max(rows, 1), n), sid=200)).cuda().to(dtype)[:rows].contiguous()
    dt = F32 if dtype == torch.float32 else BF16
    want = _reference_path(vox, x)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row: the second starts from the first call's scratch contents
        out = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
        vox._check(f(x.data_ptr(), rows, n, out.data_ptr(), dt, stream))
        got = out.item()
        # tolerance of the f32 reductions (1e-5 of the sum of magnitudes); the two paths run the same kernels, so the
        # results are in fact identical
        assert abs(got - want) <= 1e-5 * float(x.float().abs().sum())
        assert got == want
    # a smaller tensor after a larger one: stale row sums beyond `rows` must not leak into the result
    if rows > 777:
        y = x[:777].contiguous()
        out = torch.empty(1, dtype=torch.float64, device="cuda")
        vox._check(f(y.data_ptr(), 777, n, out.data_ptr(), dt, stream))
        assert out.item() == _reference_path(vox, y)


def test_noalloc_global_sum_odd_rows_unaligned_bf16(vox, port):
    """An odd row length at an address off the 16-byte grid: the scalar reduction path, on two calls in a row."""
    f = _noalloc(vox)
    rows, n = 1001, 333
    base = torch.from_numpy(port.normal((rows * n + 1,), sid=201)).cuda().to(torch.bfloat16)
    x = base[1:].view(rows, n)  # 2 bytes past a 16-byte boundary
    assert x.data_ptr() % 16 != 0
    want = _reference_path(vox, x)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        out = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
        vox._check(f(x.data_ptr(), rows, n, out.data_ptr(), BF16, stream))
        assert out.item() == want


def test_noalloc_global_sum_rejects_tensors_over_its_limit(vox):
    f = _noalloc(vox)
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    rc = f(out.data_ptr(), 262145, 16, out.data_ptr(), F32, torch.cuda.current_stream().cuda_stream)
    assert rc == -6  # VOX_CUDA_ERR_ARG, before any device work
    assert b"262144" in vox.lib.vox_cuda_last_error()
