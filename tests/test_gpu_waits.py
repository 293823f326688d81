"""The bounded-wait give-up path of the row pipelines, made to run out without a fault.

vox_cuda_test_row_stall(row, limit) tells the stage barrier of one row to expect 16 bytes more than its bulk copies
deliver: every copy lands, the barrier's phase never completes, and the warp's wait runs out after `limit` ns. The
warp must then wait (bounded) for its copies in flight, raise VOX_CUDA_DEVERR_TIMEOUT and stop; every other warp
finishes normally. The stalled row is the last one, so it is the only row left unwritten.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms: the give-up path waits twice (the stalled stage, then its copies in flight)


@pytest.fixture()
def stall(vox):
    assert vox.device_error() == 0  # nothing pending from earlier tests

    def arm(row):
        vox._check(vox.lib.vox_cuda_test_row_stall(row, LIMIT_NS))

    yield arm
    vox._check(vox.lib.vox_cuda_test_row_stall(-1, 0))
    vox.device_error()


def _rows_equal_but_last(got, want):
    got, want = got.reshape(got.shape[0], -1), want.reshape(want.shape[0], -1)
    assert np.array_equal(got[:-1], want[:-1]), "rows of the other warps must be written as in a normal run"
    assert np.isnan(got[-1]).all(), "the stalled row must stay unwritten"


def test_rmsnorm_wait_gives_up(vox, stall):
    import torch

    rows, n = 20000, 1024  # enough rows for the row pipeline
    x = vox.fill_philox(torch.empty(rows, n, device="cuda"), 1, 0, 1, seed=0, stream_id=1)
    w = vox.fill_philox(torch.empty(n, device="cuda"), 1, 1, 0.02, seed=0, stream_id=2)
    want = vox.rmsnorm(x, w, 1e-6)
    torch.cuda.synchronize()
    assert vox.device_error() == 0
    stall(rows - 1)
    out = torch.full_like(x, float("nan"))
    vox.rmsnorm(x, w, 1e-6, out=out)
    torch.cuda.synchronize()
    assert vox.device_error() & 1, "the wait for the stalled row must give up and raise the timeout bit"
    _rows_equal_but_last(out.cpu().numpy(), want.cpu().numpy())


def test_adaln_wait_gives_up(vox, stall):
    import torch

    B, T, D = 2, 2048, 1024
    bf = torch.bfloat16
    g = lambda shape, sid, s=1.0: vox.fill_philox(torch.empty(*shape, device="cuda", dtype=bf), 1, 0, s, seed=0, stream_id=sid)  # noqa: E731
    x, r = g((B, T, D), 6), g((B, T, D), 7)
    sh, sc, gt = g((B, D), 8, 0.1), g((B, D), 9, 0.1), g((B, D), 10, 0.1)
    want = vox.adaln(x, sh, sc, 1e-6, gt, r)
    torch.cuda.synchronize()
    assert vox.device_error() == 0
    stall(B * T - 1)
    out = torch.full_like(x, float("nan"))
    vox.adaln(x, sh, sc, 1e-6, gt, r, out=out)
    torch.cuda.synchronize()
    assert vox.device_error() & 1
    _rows_equal_but_last(out.float().cpu().numpy().reshape(B * T, D), want.float().cpu().numpy().reshape(B * T, D))


def test_normal_operation_restored(vox):
    """After the hook is cleared the same calls raise nothing."""
    import torch

    x = vox.fill_philox(torch.empty(20000, 1024, device="cuda"), 1, 0, 1, seed=0, stream_id=1)
    w = torch.ones(1024, device="cuda")
    vox.rmsnorm(x, w, 1e-6)
    torch.cuda.synchronize()
    assert vox.device_error() == 0
