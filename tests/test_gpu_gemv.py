"""GPU parity tests of the quantized GEMV (vox_cuda_gemv_q8 / vox_cuda_gemv_q4) through the C ABI.

Oracle: the float-activation product of Vox's GPU matvec (shaders/matmul.comp) restated in double
(oracle vo_gemv, pinned to the reference's own f32 matmul by tests/golden/gemv.npz). Bar: the rounding of an f32
dot product, |got - want| <= 1e-6 * sum_k |W[r][k] x[i][k]| (the reference's own f32 result sits within the same
bound of the exact value); bit-identical results run to run.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_gpu_parity import dev, host

pytestmark = pytest.mark.gpu


def _check(got, want, bound):
    d = np.abs(np.asarray(got, np.float64) - want)
    bad = d > 1e-6 * bound + 1e-30
    assert not bad.any(), f"{bad.sum()} of {bad.size} out of bound; worst ratio {(d / (bound + 1e-30)).max():.3e}"


def _inputs(port, rows, cols, m, q4, sid=110):
    q = port.fill_u8((rows, cols // 2), sid=sid) if q4 else port.fill_i8((rows, cols), -128, 127, sid=sid)
    s = port.uniform_arr((rows, cols // 32), 0.001, 0.05, sid=sid + 1)
    x = port.normal((m, cols), sid=sid + 2)
    b = port.normal((rows,), sid=sid + 3)
    return q, s, x, b


def _gpu(vox, q, s, x, b, q4, f16=False, out=None, accumulate=False):
    qd = dev(q) if q4 else dev(q.view(np.int8))
    sd = dev(s).to(torch.float16) if f16 else dev(s)
    fn = vox.gemv_q4 if q4 else vox.gemv_q8
    return fn(qd, sd, dev(x), bias=None if b is None else dev(b), out=out, accumulate=accumulate)


def test_gemv_golden(vox, golden):
    from oracle.oracle import port as _port

    P = _port()
    g = golden["gemv"]
    for key, q4, m, bias in (("q8_m9", False, 9, True), ("q8_m3", False, 3, True), ("q4_m3", True, 3, True),
                             ("q4_m1_nobias", True, 1, False)):
        q = g["q4" if q4 else "q8"]
        y = host(_gpu(vox, q, g["scale"], g["x"][:m], g["bias"] if bias else None, q4))
        _, bound = P.gemv(q, g["scale"], g["x"][:m], g["bias"] if bias else None, q4=q4)
        _check(y, g[key], 2 * bound)  # the reference's f32 result and ours each within 1e-6 * bound of the exact value


@pytest.mark.parametrize("q4", [False, True])
@pytest.mark.parametrize("rows,cols,m", [(4096, 4096, 1), (4096, 4096, 8), (1000, 1024, 3), (11008, 1024, 2),
                                         (1024, 11008, 5), (130, 64, 16), (7, 32, 1), (12290, 4096, 1),
                                         (12290, 4096, 4)])
def test_gemv_shapes(vox, port, q4, rows, cols, m):
    q, s, x, b = _inputs(port, rows, cols, m, q4)
    for f16, bias in ((False, b), (True, None)):
        sc = s.astype(np.float16).astype(np.float32) if f16 else s
        y = host(_gpu(vox, q, sc, x, bias, q4, f16=f16))
        want, bound = port.gemv(q, sc, x, bias, q4=q4)
        _check(y, want, bound)


@pytest.mark.parametrize("q4", [False, True])
def test_gemv_accumulate_and_determinism(vox, port, q4):
    rows, cols, m = 2048, 4096, 4
    q, s, x, b = _inputs(port, rows, cols, m, q4, sid=120)
    y0 = port.normal((m, rows), sid=125)
    out = dev(y0)
    _gpu(vox, q, s, x, b, q4, out=out, accumulate=True)
    want, bound = port.gemv(q, s, x, b, y=y0, q4=q4)
    _check(host(out), want, bound + np.abs(y0))
    r1 = host(_gpu(vox, q, s, x, b, q4))
    r2 = host(_gpu(vox, q, s, x, b, q4))
    np.testing.assert_array_equal(r1.view(np.uint32), r2.view(np.uint32))


def test_gemv_rejects_bad_shapes(vox):
    w = torch.zeros((4, 48), dtype=torch.int8, device="cuda")
    s = torch.ones((4, 1), device="cuda")
    with pytest.raises(vox.VoxCudaError) as e:
        vox.gemv_q8(w, s, torch.zeros((1, 48), device="cuda"))  # cols not a multiple of 32
    assert e.value.status == -6
    buf = torch.zeros(4 * 64 + 1, dtype=torch.int8, device="cuda")
    with pytest.raises(vox.VoxCudaError) as e:  # weights 1 byte past a 16-byte boundary
        vox.gemv_q8(buf[1:].view(4, 64), s.repeat(1, 2), torch.zeros((1, 64), device="cuda"))
    assert e.value.status == -6
