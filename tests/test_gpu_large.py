"""GPU parity at the timed sizes: every element of BASELINE config 4's Snake, and config 5's ops at 2^32 elements.

The inputs are drawn on the device (Vox's Philox4x32-10, seed 0) and copied to the host, where the oracle (the C
restatement of Vox's CPU arithmetic) runs over chunks on all host cores; every output element is compared. The f32
elementwise case has 2^32 + 8199 elements: more than 2^30 16-byte vectors, so the library splits it into two
launches (the second one's base index past 2^32) and maps a 3-element tail; the row reductions and the global sum
run over 2^20 rows of 4096 (2^32 elements). Bars as the other parity tests: bit-exact for add / mul, the fixed-order
row reductions and the global sum; 1e-5 relative for f32 GELU and Snake (1e-6 |x| where x + sin^2/alpha nearly
cancels), 1e-2 for bf16 GELU; the Kokoro Snake bit-exact.
"""

from __future__ import annotations

import concurrent.futures as cf
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1
CHUNK = 1 << 25  # elements compared per step on the host


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _par(fn, n, step):
    """fn(lo, hi) over [0, n) in steps of `step`, on all host cores (the C oracle releases the GIL)."""
    with cf.ThreadPoolExecutor(THREADS) as ex:
        list(ex.map(lambda lo: fn(lo, min(n, lo + step)), range(0, n, step)))


def _host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _wide(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def test_snake_config4_every_element(vox, port):
    """HiFT and Kokoro Snake on x [16, 512, 24000] f32 channel-major, all 196,608,000 elements."""
    B, C, T = 16, 512, 24000
    x = vox.fill_philox(torch.empty(B, C, T, device="cuda"), 1, 0, 1, seed=0, stream_id=120)
    al = vox.fill_philox(torch.empty(C, device="cuda"), 0, 0.2, 2.0, seed=0, stream_id=121)
    xh, ah = _host(x).reshape(-1), _host(al)
    for kind in (vox.SNAKE_HIFT, vox.SNAKE_KOKORO):
        got = _host(vox.snake(x, al, kind)).reshape(-1)
        want = np.empty_like(xh)
        # one batch [C][T] per oracle call, so the channel the oracle derives from the element index, (i / T) % C, is
        # the element's own channel
        _par(lambda lo, hi: _run_rows(port, xh, ah, want, lo, hi, C, T, kind), B * C, C)
        if kind == vox.SNAKE_KOKORO:
            bad = got.view(np.uint32) != want.view(np.uint32)
        else:
            bad = np.abs(got - want) > np.maximum(1e-5 * np.abs(want), 1e-6 * np.abs(xh)) + 1e-30
        assert not bad.any(), f"kind {kind}: {int(bad.sum())} of {bad.size} elements differ, first at {int(np.argmax(bad))}"
        del got, want


def _run_rows(port, xh, ah, want, lo, hi, C, T, kind):
    """The oracle's Snake on channel rows [lo, hi) (lo a multiple of C)."""
    a, b = lo * T, hi * T
    port.L.vo_snake(_p(xh[a:b]), _p(ah), None, _p(want[a:b]), b - a, C, T, kind)


def test_cfg5_f32_past_the_launch_split(vox, port):
    """add / mul / GELU on 2^32 + 8199 f32 elements (two launches and a tail); row sum / max / L2 and the global sum
    over 2^20 rows of 4096."""
    n = (1 << 32) + 8199
    a = vox.fill_philox(torch.empty(n, device="cuda"), 1, 0, 1, seed=0, stream_id=16)
    b = vox.fill_philox(torch.empty(n, device="cuda"), 1, 0, 1, seed=0, stream_id=18)
    y = torch.empty_like(a)
    for op in ("add", "mul", "gelu"):
        if op == "add":
            vox.add(a, b, out=y)
        elif op == "mul":
            vox.mul(a, b, out=y)
        else:
            vox.gelu(a, vox.GELU_ERF, out=y)
        torch.cuda.synchronize()
        for lo in list(range(0, n, CHUNK)):
            hi = min(n, lo + CHUNK)
            ah, gh = a[lo:hi].cpu().numpy(), y[lo:hi].cpu().numpy()
            want = np.empty_like(ah)
            if op == "gelu":
                _par(lambda s, e: port.L.vo_gelu_erf(_p(ah[s:e]), _p(want[s:e]), e - s), hi - lo, 1 << 20)
                bad = np.abs(gh - want) > 1e-5 * np.maximum(np.abs(want), 1.0)
            else:
                bh = b[lo:hi].cpu().numpy()
                fn = port.L.vo_add if op == "add" else port.L.vo_mul
                _par(lambda s, e: fn(_p(ah[s:e]), _p(bh[s:e]), _p(want[s:e]), e - s), hi - lo, 1 << 22)
                bad = gh.view(np.uint32) != want.view(np.uint32)
            assert not bad.any(), f"{op}: {int(bad.sum())} elements differ in [{lo}, {hi})"
    del y, b
    rows = 1 << 20
    x = a[: rows * 4096].view(rows, 4096)
    out = {k: _host(vox.row_reduce(x, k)) for k in (vox.REDUCE_SUM, vox.REDUCE_MAX, vox.REDUCE_L2)}
    slots = _host(vox.global_sum_partials(x, 0, rows))
    total = _host(vox.global_sum_finish(torch.from_numpy(slots).cuda()))[0]
    step_rows = CHUNK // 4096
    want = {k: np.empty(rows, np.float32) for k in out}
    for r0 in range(0, rows, step_rows):
        xh = x[r0:r0 + step_rows].cpu().numpy()
        for k in out:
            w = want[k][r0:r0 + step_rows]
            _par(lambda s, e: port.L.vo_row_reduce_ordered(_p(xh[s:e]), _p(w[s:e]), e - s, 4096, k, 4), len(xh), 256)
    for k in out:
        np.testing.assert_array_equal(out[k].view(np.uint32), want[k].view(np.uint32))
    np.testing.assert_array_equal(slots, port.global_sum_slots(want[vox.REDUCE_SUM], 0, rows))
    assert total == port.global_sum_finish(slots)


def test_cfg5_bf16_2pow32(vox, port):
    """add / mul / GELU and row sum / max / L2 on 2^32 bf16 elements (rows of 4096)."""
    n = 1 << 32
    a = vox.fill_philox(torch.empty(n, dtype=torch.bfloat16, device="cuda"), 1, 0, 1, seed=0, stream_id=17)
    b = vox.fill_philox(torch.empty(n, dtype=torch.bfloat16, device="cuda"), 1, 0, 1, seed=0, stream_id=19)
    y = torch.empty_like(a)
    for op in ("add", "mul", "gelu"):
        if op == "add":
            vox.add(a, b, out=y)
        elif op == "mul":
            vox.mul(a, b, out=y)
        else:
            vox.gelu(a, vox.GELU_ERF, out=y)
        torch.cuda.synchronize()
        for lo in range(0, n, CHUNK):
            hi = min(n, lo + CHUNK)
            ah = _wide(a[lo:hi].view(torch.int16).cpu().numpy().view(np.uint16))
            gh = y[lo:hi].view(torch.int16).cpu().numpy().view(np.uint16)
            want = np.empty_like(ah)
            if op == "gelu":
                _par(lambda s, e: port.L.vo_gelu_erf(_p(ah[s:e]), _p(want[s:e]), e - s), hi - lo, 1 << 20)
            else:
                bh = _wide(b[lo:hi].view(torch.int16).cpu().numpy().view(np.uint16))
                fn = port.L.vo_add if op == "add" else port.L.vo_mul
                _par(lambda s, e: fn(_p(ah[s:e]), _p(bh[s:e]), _p(want[s:e]), e - s), hi - lo, 1 << 22)
            wb = np.empty(hi - lo, np.uint16)
            _par(lambda s, e: port.L.vo_f32_to_bf16_n(_p(want[s:e]), _p(wb[s:e]), e - s), hi - lo, 1 << 22)
            if op == "gelu":
                bad = np.abs(_wide(gh) - _wide(wb)) > 1e-2 * np.maximum(np.abs(_wide(wb)), 1.0)
            else:
                bad = gh != wb
            assert not bad.any(), f"{op} bf16: {int(bad.sum())} elements differ in [{lo}, {hi})"
    del y, b
    rows = n // 4096
    x = a.view(rows, 4096)
    out = {k: _host(vox.row_reduce(x, k)) for k in (vox.REDUCE_SUM, vox.REDUCE_MAX, vox.REDUCE_L2)}
    step_rows = CHUNK // 4096
    for r0 in range(0, rows, step_rows):
        xh = _wide(x[r0:r0 + step_rows].view(torch.int16).cpu().numpy().view(np.uint16))
        for k in out:
            w = np.empty(len(xh), np.float32)
            _par(lambda s, e: port.L.vo_row_reduce_ordered(_p(xh[s:e]), _p(w[s:e]), e - s, 4096, k, 8), len(xh), 256)
            np.testing.assert_array_equal(out[k][r0:r0 + step_rows].view(np.uint32), w.view(np.uint32))
