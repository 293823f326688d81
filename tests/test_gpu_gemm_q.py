"""GPU parity tests of the quantized prefill GEMM (vox_cuda_gemm_q8 / vox_cuda_gemm_q4) through the C ABI.

Oracle: the float-activation product restated in double (oracle vo_gemv, pinned to the reference's own f32 matmul by
tests/golden/gemv.npz, whose m = 9 case is the reference's dequantise-then-matmul path for m > 8). The kernel computes
in f16 on the tensor cores: x and code * scale each keep 11 significant bits, so every product is within 2^-10 of
exact and the sum within |got - want| <= 1.5e-3 * sum_k |W[r][k] x[i][k]| of the exact value; bit-identical results
run to run.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_gpu_parity import dev, host

pytestmark = pytest.mark.gpu

TOL = 1.5e-3


def _check(got, want, bound):
    d = np.abs(np.asarray(got, np.float64) - want)
    bad = d > TOL * bound + 1e-30
    assert not bad.any(), f"{bad.sum()} of {bad.size} out of bound; worst ratio {(d / (bound + 1e-30)).max():.3e}"


def _inputs(port, rows, cols, m, q4, sid=210):
    q = port.fill_u8((rows, cols // 2), sid=sid) if q4 else port.fill_i8((rows, cols), -128, 127, sid=sid)
    s = port.uniform_arr((rows, cols // 32), 0.001, 0.05, sid=sid + 1)
    x = port.normal((m, cols), sid=sid + 2)
    b = port.normal((rows,), sid=sid + 3)
    return q, s, x, b


def _gpu(vox, q, s, x, b, q4, f16=False, out=None, accumulate=False):
    qd = dev(q) if q4 else dev(q.view(np.int8))
    sd = dev(s).to(torch.float16) if f16 else dev(s)
    fn = vox.gemm_q4 if q4 else vox.gemm_q8
    return fn(qd, sd, dev(x), bias=None if b is None else dev(b), out=out, accumulate=accumulate)


def test_gemm_q_golden(vox, golden):
    """The reference's own matmul output (Q8 with m = 9: its dequantise-then-f32 path; Q4 with m = 3)."""
    from oracle.oracle import port as _port

    P = _port()
    g = golden["gemv"]
    for key, q4, m in (("q8_m9", False, 9), ("q4_m3", True, 3)):
        q = g["q4" if q4 else "q8"]
        y = host(_gpu(vox, q, g["scale"], g["x"][:m], g["bias"], q4))
        _, bound = P.gemv(q, g["scale"], g["x"][:m], g["bias"], q4=q4)
        _check(y, g[key], bound)


@pytest.mark.parametrize("q4", [False, True])
@pytest.mark.parametrize("rows,cols,m", [(4096, 4096, 512), (1000, 1024, 130), (300, 96, 9), (257, 4064, 200), (12288, 1024, 64),
                                         (12288, 1024, 512), (10000, 512, 520), (20000, 512, 300)])
def test_gemm_q_shapes(vox, port, q4, rows, cols, m, monkeypatch):
    """Tile edges in every dimension (rows and m not multiples of 256 / 128, cols an odd number of 32-blocks), both
    forms (one pass; two passes: W to f16, then the f16 GEMM, the default from 256 rows of x), and every one-pass work
    schedule on 148 SMs: one partial wave cut into K-ranges (4096 x 512: 64 tiles, 2 pieces each), whole
    tiles plus K-range pieces of the tail (12288 x 512: 192 tiles, the last 44 in 3 pieces; 10000 x 520: 200 tiles,
    the last 52 in 2 pieces with ragged rows and columns), whole tiles only (20000 x 300: 237 tiles), tiny K unsplit."""
    q, s, x, b = _inputs(port, rows, cols, m, q4)
    for f16, bias in ((False, b), (True, None)):
        sc = s.astype(np.float16).astype(np.float32) if f16 else s
        want, bound = port.gemv(q, sc, x, bias, q4=q4)
        for two in ("0", "1"):  # one pass (codes converted in the GEMM) and two passes (f16 W, then the f16 GEMM)
            monkeypatch.setenv("VOX_CUDA_GEMMQ_TWOPASS", two)
            y = host(_gpu(vox, q, sc, x, bias, q4, f16=f16))
            _check(y, want, bound)
    assert vox.device_error() == 0


@pytest.mark.parametrize("q4", [False, True])
def test_gemm_q_accumulate_and_determinism(vox, port, q4):
    rows, cols, m = 2048, 2048, 100
    q, s, x, b = _inputs(port, rows, cols, m, q4, sid=220)
    y0 = port.normal((m, rows), sid=225)
    out = dev(y0)
    _gpu(vox, q, s, x, b, q4, out=out, accumulate=True)
    want, bound = port.gemv(q, s, x, b, y=y0, q4=q4)
    _check(host(out), want, bound + np.abs(y0))
    r1 = host(_gpu(vox, q, s, x, b, q4))
    r2 = host(_gpu(vox, q, s, x, b, q4))
    np.testing.assert_array_equal(r1.view(np.uint32), r2.view(np.uint32))


@pytest.mark.parametrize("q4", [False, True])
def test_gemm_q_split_schedule_matches_whole_tiles(vox, port, q4, monkeypatch):
    """The one-pass K-range pieces and their fixed-order sum agree with whole tiles (VOX_CUDA_GEMMQ_SPLIT=0) and the
    two-pass form to the oracle's bound, each accumulates into y, and each repeats bit for bit."""
    rows, cols, m = 12288, 1024, 512
    q, s, x, b = _inputs(port, rows, cols, m, q4, sid=230)
    y0 = port.normal((m, rows), sid=235)
    want, bound = port.gemv(q, s, x, b, y=y0, q4=q4)
    for two, split in (("0", "1"), ("0", "0"), ("1", "1")):
        monkeypatch.setenv("VOX_CUDA_GEMMQ_TWOPASS", two)
        monkeypatch.setenv("VOX_CUDA_GEMMQ_SPLIT", split)
        out = dev(y0)
        _gpu(vox, q, s, x, b, q4, out=out, accumulate=True)
        _check(host(out), want, bound + np.abs(y0))
        r1 = host(_gpu(vox, q, s, x, b, q4))
        r2 = host(_gpu(vox, q, s, x, b, q4))
        np.testing.assert_array_equal(r1.view(np.uint32), r2.view(np.uint32))
    assert vox.device_error() == 0
