"""The cross-GPU global sum in one library call (vox_cuda_global_sum over a vox_cuda_comm, NCCL loaded at run time).

On one GPU: a communicator of one rank, the result equal to the two-step path (partials + fold). On two or more GPUs
(skipped otherwise): two processes, one per GPU, each holding a shard of the same global tensor; both get the bits of
the one-GPU sum. NVLS is off (NCCL_NVLS_ENABLE=0) in the child processes, and every wait is bounded by the
library's deadline.
"""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_global_sum_one_rank_comm_matches_two_step_path(vox):
    R, n = 3000, 4096
    x = vox.fill_philox(torch.empty(R, n, device="cuda"), 1, 0, 1, seed=0, stream_id=300)
    want = vox.global_sum_finish(vox.global_sum_partials(x, 0, R)).item()
    comm = vox.Comm(vox.Comm.unique_id(), 1, 0)
    try:
        got = vox.global_sum_comm(x, 0, R, comm).item()
        comm.wait(timeout_ms=10000)
        assert got == want
        assert vox.global_sum_comm(x, 0, R, None).item() == want  # no communicator: the single-GPU sum
    finally:
        comm.close()


_CHILD = textwrap.dedent("""
    import os, sys, time, torch
    sys.path.insert(0, os.environ["VOX_ROOT"])
    import vox_b200 as vox
    from vox_b200.shard import shard_rows
    rank, world, uid_path = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    torch.cuda.set_device(rank)
    if rank == 0:
        open(uid_path + ".tmp", "wb").write(vox.Comm.unique_id())
        os.replace(uid_path + ".tmp", uid_path)
    t0 = time.time()
    while not os.path.exists(uid_path):
        if time.time() - t0 > 60:
            sys.exit(3)
        time.sleep(0.05)
    comm = vox.Comm(open(uid_path, "rb").read(), world, rank, timeout_ms=60000)
    R, n = 3360, 4096
    r0, rows = shard_rows(R, world, rank)
    x = vox.fill_philox(torch.empty(rows, n, device="cuda"), 1, 0, 1, seed=0, stream_id=301, counter0=r0 * n)
    got = vox.global_sum_comm(x, r0, R, comm)
    comm.wait(timeout_ms=30000)
    print(repr(got.item()), flush=True)
    comm.close()
""")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_global_sum_two_ranks_bitwise_equals_one_gpu(vox, tmp_path):
    R, n = 3360, 4096
    x = vox.fill_philox(torch.empty(R, n, device="cuda"), 1, 0, 1, seed=0, stream_id=301)
    want = vox.global_sum_finish(vox.global_sum_partials(x, 0, R)).item()
    env = dict(os.environ, VOX_ROOT=str(ROOT), NCCL_NVLS_ENABLE="0")
    script = tmp_path / "child.py"
    script.write_text(_CHILD)
    uid = str(tmp_path / "uid")
    procs = [subprocess.Popen([sys.executable, str(script), str(r), "2", uid], env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                              text=True) for r in range(2)]
    outs = [p.communicate(timeout=240) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, e[-2000:]
    assert [float(o.strip().splitlines()[-1]) for o, _ in outs] == [want, want]
