"""Multi-process (gloo, world_size 2) checks of the sharded path on CPU: every rank runs the
oracle on its own shard, the shards reassemble into the single-process result, and the
timing reduction used by bench.py (MAX over ranks) behaves.  No GPU involved."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from gdn.shard import batch_shard, head_shard, seq_shard


def test_batch_shard_covers_everything():
    for B in (0, 1, 7, 64, 512):
        for world in (1, 2, 3, 8):
            spans = [batch_shard(B, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def test_seq_shard_rebases_and_covers():
    cu = [0, 4096 * 1, 4096 * 2, 4096 * 3, 4096 * 4]
    parts = [seq_shard(cu, 2, r) for r in range(2)]
    assert parts[0][:4] == (0, 2, 0, 8192) and parts[1][:4] == (2, 4, 8192, 16384)
    assert parts[1][4] == [0, 4096, 8192]
    cu2 = [0, 5, 5, 100, 130, 131]
    for world in (1, 2, 3, 4):
        ps = [seq_shard(cu2, world, r) for r in range(world)]
        assert ps[0][0] == 0 and ps[-1][1] == 5
        assert all(ps[i][1] == ps[i + 1][0] for i in range(world - 1))


def test_head_shard_groups_and_constraints():
    # the reference family (4 q/k heads, 8 v-heads): 1, 2, 4 or 8 ranks, decode and prefill alike
    for world in (1, 2, 4, 8):
        for prefill in (False, True):
            parts = [head_shard(4, 8, world, r, prefill=prefill) for r in range(world)]
            assert parts[0][2] == 0 and parts[-1][3] == 8
            assert all(parts[i][3] == parts[i + 1][2] for i in range(world - 1))  # v-heads tile [0, 8)
            for a0, a1, b0, b1 in parts:
                # every v-head of the rank reads one of the rank's q/k heads, in grouped order
                assert all(a0 <= hv // 2 < a1 for hv in range(b0, b1))
                assert (b1 - b0) % (a1 - a0) == 0
    assert head_shard(4, 8, 8, 5) == (2, 3, 5, 6)  # v-head 5 reads q/k head 2
    assert head_shard(4, 8, 2, 1, prefill=True) == (2, 4, 4, 8)
    assert head_shard(16, 32, 4, 3, prefill=True) == (12, 16, 24, 32)
    with pytest.raises(ValueError):
        head_shard(4, 8, 3, 0)  # 3 does not divide 8 v-heads
    with pytest.raises(ValueError):
        head_shard(3, 6, 2, 0)  # 3 v-heads per rank: one and a half groups of 2
    with pytest.raises(ValueError):
        head_shard(2, 12, 3, 0)  # 4 v-heads per rank do not divide a group of 6


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch

        from oracle import oracle
        from tests.golden import inputs as gi

        # decode: shard a batch of 6
        d = gi.decode_inputs(6, seed=3)
        s0, s1 = batch_shard(6, world, rank)
        o, st = oracle.decode(*(d[x][s0:s1] for x in ("q", "k", "v", "state")), d["A_log"], d["a"][s0:s1],
                              d["dt_bias"], d["b"][s0:s1], d["scale"], threads=1)
        dec = [None] * world
        dist.all_gather_object(dec, (o, st))
        # prefill: shard 4 sequences by tokens
        lens = [40, 70, 3, 90]
        p = gi.prefill_inputs(lens, seed=4)
        q0, q1, t0, t1, lcu = seq_shard(p["cu_seqlens"], world, rank)
        po, ps = oracle.prefill(p["q"][t0:t1], p["k"][t0:t1], p["v"][t0:t1], p["state"][q0:q1], p["A_log"],
                                p["a"][t0:t1], p["dt_bias"], p["b"][t0:t1], np.array(lcu), p["scale"], threads=1)
        pre = [None] * world
        dist.all_gather_object(pre, (po, ps))
        # one sequence split by v-head groups (fewer sequences than ranks): decode of the reference
        # family (4 q/k heads, 8 v-heads) and prefill of the 16 / 32 family
        h0, h1, v0, v1 = head_shard(4, 8, world, rank)
        hd = gi.decode_inputs(1, seed=5)
        ho = oracle.decode(hd["q"][:, :, h0:h1], hd["k"][:, :, h0:h1], hd["v"][:, :, v0:v1], hd["state"][:, v0:v1],
                           hd["A_log"][v0:v1], hd["a"][:, :, v0:v1], hd["dt_bias"][v0:v1], hd["b"][:, :, v0:v1],
                           hd["scale"], threads=1)
        hp = gi.prefill_inputs([150], seed=6, h=16, hv=32)
        h0, h1, v0, v1 = head_shard(16, 32, world, rank, prefill=True)
        hpo = oracle.prefill(hp["q"][:, h0:h1], hp["k"][:, h0:h1], hp["v"][:, v0:v1], hp["state"][:, v0:v1],
                             hp["A_log"][v0:v1], hp["a"][:, v0:v1], hp["dt_bias"][v0:v1], hp["b"][:, v0:v1],
                             hp["cu_seqlens"], hp["scale"], threads=1)
        # prefill of the reference family (4 q/k heads, 8 v-heads) split by v-heads
        rp = gi.prefill_inputs([130], seed=7)
        h0, h1, v0, v1 = head_shard(4, 8, world, rank, prefill=True)
        rpo = oracle.prefill(rp["q"][:, h0:h1], rp["k"][:, h0:h1], rp["v"][:, v0:v1], rp["state"][:, v0:v1],
                             rp["A_log"][v0:v1], rp["a"][:, v0:v1], rp["dt_bias"][v0:v1], rp["b"][:, v0:v1],
                             rp["cu_seqlens"], rp["scale"], threads=1)
        heads = [None] * world
        dist.all_gather_object(heads, (ho, hpo, rpo))
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((dec, pre, heads, float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_sharded_oracle_matches_single_process():
    from oracle import oracle
    from tests.golden import inputs as gi

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    dec, pre, heads, tmax = q.get()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert tmax == float(world)
    d = gi.decode_inputs(6, seed=3)
    fo, fs = oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], d["scale"])
    assert np.array_equal(np.concatenate([x[0] for x in dec]), fo)
    assert np.array_equal(np.concatenate([x[1] for x in dec]), fs)
    p = gi.prefill_inputs([40, 70, 3, 90], seed=4)
    po, ps = oracle.prefill(p["q"], p["k"], p["v"], p["state"], p["A_log"], p["a"], p["dt_bias"], p["b"],
                            p["cu_seqlens"], p["scale"])
    assert np.array_equal(np.concatenate([x[0] for x in pre]), po)
    assert np.array_equal(np.concatenate([x[1] for x in pre]), ps)

    hd = gi.decode_inputs(1, seed=5)
    fo, fs = oracle.decode(hd["q"], hd["k"], hd["v"], hd["state"], hd["A_log"], hd["a"], hd["dt_bias"], hd["b"],
                           hd["scale"])
    assert np.array_equal(np.concatenate([x[0][0] for x in heads], axis=2), fo)
    assert np.array_equal(np.concatenate([x[0][1] for x in heads], axis=1), fs)
    hp = gi.prefill_inputs([150], seed=6, h=16, hv=32)
    po, ps = oracle.prefill(hp["q"], hp["k"], hp["v"], hp["state"], hp["A_log"], hp["a"], hp["dt_bias"], hp["b"],
                            hp["cu_seqlens"], hp["scale"])
    assert np.array_equal(np.concatenate([x[1][0] for x in heads], axis=1), po)
    assert np.array_equal(np.concatenate([x[1][1] for x in heads], axis=1), ps)
    rp = gi.prefill_inputs([130], seed=7)
    po, ps = oracle.prefill(rp["q"], rp["k"], rp["v"], rp["state"], rp["A_log"], rp["a"], rp["dt_bias"], rp["b"],
                            rp["cu_seqlens"], rp["scale"])
    assert np.array_equal(np.concatenate([x[2][0] for x in heads], axis=1), po)
    assert np.array_equal(np.concatenate([x[2][1] for x in heads], axis=1), ps)
