"""Partitioning of independent work across ranks (one process per GPU).

Decode batch elements and prefill sequences are independent units of this path
(reference/gdn_prefill_ref.py:56-89 loops over sequences with no exchange), so a
multi-GPU run splits them into contiguous shards and needs no collective on the
data path.  These helpers compute each rank's shard on the host.
"""
from __future__ import annotations

from typing import Sequence, Tuple


def batch_shard(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of `batch` elements owned by `rank` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError("need world > 0, 0 <= rank < world, batch >= 0")
    base, rem = divmod(batch, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def seq_shard(cu_seqlens: Sequence[int], world: int, rank: int):
    """Shard packed sequences by token count.

    Returns (seq_start, seq_stop, tok_start, tok_stop, local_cu) where local_cu is the
    rank's cu_seqlens rebased to 0.  Sequences are assigned greedily in order so that
    each rank's token count is close to total / world.
    """
    cu = [int(x) for x in cu_seqlens]
    n = len(cu) - 1
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError("bad world/rank/cu_seqlens")
    total = cu[-1] - cu[0] if n > 0 else 0
    bounds = [0]
    for r in range(1, world):
        target = cu[0] + total * r / world
        s = bounds[-1]
        while s < n and cu[s + 1] <= target + 1e-9:
            s += 1
        bounds.append(s)
    bounds.append(n)
    s0, s1 = bounds[rank], bounds[rank + 1]
    t0, t1 = cu[s0], cu[s1]
    local = [x - t0 for x in cu[s0:s1 + 1]]
    return s0, s1, t0, t1, local
