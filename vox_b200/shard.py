"""Row sharding of the multi-GPU sweep, aligned to the slots of the deterministic global sum.

The global tensor [R][n] is split into ``GLOBAL_SUM_SLOTS`` = 840 = lcm(1..8) slots, slot s = rows
[floor(s*R/840), floor((s+1)*R/840)). Rank k of a world of size W (W divides 840) owns slots
[k*840/W, (k+1)*840/W), i.e. the contiguous rows [floor(k*R/W), floor((k+1)*R/W)). Each shard is therefore a whole
number of slots, which is what ``vox_cuda_global_sum_partials`` requires.
"""

from __future__ import annotations

GLOBAL_SUM_SLOTS = 840


def slot_begin(s: int, total_rows: int) -> int:
    return (s * total_rows) // GLOBAL_SUM_SLOTS


def shard_rows(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, rows) of rank's shard; world must divide 840 (every world size 1..8 does)."""
    if world < 1 or GLOBAL_SUM_SLOTS % world:
        raise ValueError(f"world size {world} does not divide {GLOBAL_SUM_SLOTS}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    s0 = rank * GLOBAL_SUM_SLOTS // world
    s1 = (rank + 1) * GLOBAL_SUM_SLOTS // world
    r0, r1 = slot_begin(s0, total_rows), slot_begin(s1, total_rows)
    return r0, r1 - r0
