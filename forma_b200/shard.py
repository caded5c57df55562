"""Work partitioning across ranks (one process per GPU).

Every sharded workload of the dense-op path splits one leading dimension into
contiguous, nearly equal blocks: rows of a reduction, images of a batch, or
(batch, head) pairs of attention.  No data moves between ranks except the
single 8-byte all-reduce of a global sum.
"""

from __future__ import annotations


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of `rank`'s block of `total` units over `world` ranks;
    the first `total % world` ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid world/rank")
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)
