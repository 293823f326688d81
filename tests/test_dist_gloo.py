"""Multi-process host logic of the sharded sweep on CPU (gloo ranks, no GPU): the row sharding of vox_b200.shard,
the 840-slot partials of every shard, one all-reduce, and the fixed-order fold give a global sum that is bitwise the
single-shard result for every world size; a rank that fails before the collective is detected by the others as an
error, not a hang. The slot arithmetic is the oracle's restatement of the CUDA kernels' order."""

from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]

R_ROWS, N_COLS = 2000, 64


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, mode: str, q) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from oracle.oracle import port as oracle_port
        from vox_b200.shard import shard_rows

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        P = oracle_port()
        r0, rows = shard_rows(R_ROWS, world, rank)
        # each rank draws its own rows from the counter stream of the global tensor (no data broadcast)
        x = P.fill(rows * N_COLS, 1, 0.0, 1.0, seed=3, sid=1, c0=r0 * N_COLS).reshape(rows, N_COLS)
        slots = torch.from_numpy(P.global_sum_slots(P.row_reduce(x, 0), r0, R_ROWS))
        if mode == "fail" and rank == world - 1:
            raise RuntimeError("injected failure before the collective")
        dist.all_reduce(slots, op=dist.ReduceOp.SUM)
        total = P.global_sum_finish(slots.numpy())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", total))
    except Exception as e:  # reported to the parent, never swallowed
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=2)}"))


def _run(world: int, mode: str = "ok"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out)


def _single_rank_total() -> float:
    sys.path.insert(0, str(ROOT))
    from oracle.oracle import port as oracle_port

    P = oracle_port()
    x = P.fill(R_ROWS * N_COLS, 1, 0.0, 1.0, seed=3, sid=1).reshape(R_ROWS, N_COLS)
    return P.global_sum_finish(P.global_sum_slots(P.row_reduce(x, 0), 0, R_ROWS))


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_global_sum_is_bitwise_world_size_invariant(world):
    want = _single_rank_total()
    out = _run(world)
    assert all(status == "ok" for _, status, _ in out), out
    assert all(total == want for _, _, total in out), (out, want)


def test_rank_failure_before_collective_is_reported():
    out = _run(2, mode="fail")
    status = {r: s for r, s, _ in out}
    assert status[1] == "error"  # the failing rank reports its own exception
    assert status[0] == "error"  # the surviving rank's collective fails (peer gone) instead of hanging
