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


def head_shard(num_qk_heads: int, num_v_heads: int, world: int, rank: int, prefill: bool = False):
    """Split the heads of a call over ranks, for calls with fewer independent sequences (or batch
    elements) than ranks.  Each rank takes HV / world consecutive v-heads and the q/k heads they
    read (v-head hv reads q/k head hv // (HV // H)); v-heads never exchange anything, so neither do
    the shards.  A rank holds whole q/k head groups, or part of one group (then it reads one q/k
    head that another rank reads too: an input, copied, not exchanged).

    Returns (qk_start, qk_stop, v_start, v_stop).  The rank runs the path on
    q[..., qk_start:qk_stop, :], k likewise, and v, a, b, A_log, dt_bias and the state sliced to
    [v_start, v_stop) along their head dimension; its local call then has HV / world v-heads
    reading qk_stop - qk_start q/k heads in the same grouped order.

    world must divide HV, and each rank's v-heads must be whole groups or an equal part of one
    group; otherwise ValueError.  The reference's 4 q/k heads and 8 v-heads split over 2, 4 or 8
    ranks (8: one v-head and its q/k head per rank), so one long sequence can use every GPU of a
    box.  Decode and prefill take the same splits (prefill is accepted and changes nothing).
    """
    H, HV = int(num_qk_heads), int(num_v_heads)
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("need world > 0 and 0 <= rank < world")
    if H <= 0 or HV % H:
        raise ValueError(f"v-heads ({HV}) must be a multiple of q/k heads ({H})")
    if HV % world:
        raise ValueError(f"{world} ranks cannot split {HV} v-heads into equal groups")
    group = HV // H  # v-heads per q/k head
    hv = HV // world
    v0, v1 = rank * hv, (rank + 1) * hv
    if hv >= group:
        if hv % group:
            raise ValueError(f"{hv} v-heads per rank would split a group of {group}")
        return v0 // group, v1 // group, v0, v1
    if group % hv:
        raise ValueError(f"{hv} v-heads per rank do not divide a group of {group}")
    return v0 // group, v0 // group + 1, v0, v1
