"""Prefill parity on the GPU: the CUDA path (through the C ABI) against the CPU oracle
and the reference's golden outputs.  Cases follow the reference's own prefill tests
(in-chunk, multi-chunk, ragged tails, multi-sequence, initial state) plus the
benchmark configurations at full size."""
import numpy as np
import pytest
import torch

import gdn
from oracle import oracle
from tests import util
from tests.golden import check, inputs as gi

pytestmark = pytest.mark.gpu


def _oracle(inp):
    return oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                          inp["b"], inp["cu_seqlens"], inp["scale"])


def _run_and_check(inp, cu_dtype=torch.int32):
    out, ns = gdn.prefill.run(*util.prefill_args(inp, cu_dtype=cu_dtype))
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    err = util.check_out(util.bits(out), ro)
    rel = util.check_state(ns.cpu().numpy(), rs)
    return err, rel


CASES = [
    ([32], False), ([64], False), ([128], False), ([256], False),
    ([31], False), ([65], False), ([127], False),
    ([64, 64], False), ([32, 96], False), ([64, 128], False),
    ([64], True), ([128], True), ([64, 128], True),
    ([1], True), ([2, 3, 1, 63, 129], True), ([1000], True),
]


@pytest.mark.parametrize("lens,with_state", CASES, ids=[f"{'-'.join(map(str, l))}{'-h0' if s else ''}"
                                                         for l, s in CASES])
def test_prefill_matches_oracle(lens, with_state):
    inp = gi.prefill_inputs(lens, seed=sum(lens) + 7 * len(lens), with_state=with_state)
    _run_and_check(inp)


@pytest.mark.parametrize("name,fx", check.fixtures("prefill"), ids=[n for n, _ in check.fixtures("prefill")])
def test_prefill_matches_reference_golden(name, fx):
    inp = check.regen(fx)
    out, ns = gdn.prefill.run(*util.prefill_args(inp))
    torch.cuda.synchronize()
    check.compare(fx, "out", util.bits(out), atol=util.OUT_ATOL, rtol=util.OUT_RTOL, proj_rtol=1e-2)
    # state: the bar is rel-L2 1e-3; projections on +-1 vectors bound it the same way
    check.compare(fx, "state", ns.cpu().numpy(), atol=1e-3, rtol=1e-2, proj_rtol=1e-3)


@pytest.mark.parametrize("lens", [[70, 33, 129], [1, 24, 25, 3, 200, 0, 17] * 6, [6] * 40, [5, 20]],
                         ids=["mma_sync_scan", "short_path_persistent", "short_rec", "only_short"])
def test_prefill_int64_cu_seqlens(lens):
    """int64 cu_seqlens give bit-identical results to int32 on every route (chunked, short path with
    the chunk table and persistent grids, token recurrence, single-launch short kernel)."""
    inp = gi.prefill_inputs(lens, seed=21)
    o32, s32 = gdn.prefill.run(*util.prefill_args(inp, cu_dtype=torch.int32))
    o64, s64 = gdn.prefill.run(*util.prefill_args(inp, cu_dtype=torch.int64))
    torch.cuda.synchronize()
    assert torch.equal(o32, o64) and torch.equal(s32, s64)


def test_prefill_cpu_cu_seqlens_accepted():
    inp = gi.prefill_inputs([50, 14], seed=22)
    args = list(util.prefill_args(inp))
    ref = gdn.prefill.run(*args)
    args[8] = args[8].cpu()
    got = gdn.prefill.run(*args)
    torch.cuda.synchronize()
    assert torch.equal(ref[0], got[0]) and torch.equal(ref[1], got[1])


def test_prefill_zero_length_sequences():
    inp = gi.prefill_inputs([40, 0, 70, 0], seed=23)
    out, ns = gdn.prefill.run(*util.prefill_args(inp))
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)
    assert torch.count_nonzero(ns[1]) == 0 and torch.count_nonzero(ns[3]) == 0


def test_prefill_uncovered_tokens_are_zero():
    """Tokens outside [cu[0], cu[N]) keep a zero output (the reference zero-initialises output)."""
    inp = gi.prefill_inputs([100], seed=24)
    T = 100
    inp["cu_seqlens"] = np.array([10, 80], np.int32)
    out, ns = gdn.prefill.run(*util.prefill_args(inp))
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)
    assert torch.count_nonzero(out[:10]) == 0 and torch.count_nonzero(out[80:]) == 0
    assert out.shape[0] == T


def test_prefill_t1_matches_decode():
    d = gi.decode_inputs(6, seed=25)
    q, k, v, st, A_log, a, dt_bias, b, scale = util.decode_args(d)
    od, sd = gdn.decode.run(q, k, v, st, A_log, a, dt_bias, b, scale)
    cu = torch.arange(7, dtype=torch.int32, device="cuda")
    op, sp = gdn.prefill.run(q.view(6, 4, 128), k.view(6, 4, 128), v.view(6, 8, 128), st, A_log, a.view(6, 8),
                             dt_bias, b.view(6, 8), cu, scale)
    torch.cuda.synchronize()
    util.check_out(util.bits(op), util.bits(od.view(6, 8, 128)), atol=1e-3, rtol=1e-2)
    util.check_state(sp.cpu().numpy(), sd.cpu().numpy(), rel_l2=1e-4)


@pytest.mark.parametrize("lens", [[90, 200], [1, 24, 25, 3, 200, 0, 17] * 6, [6] * 40, [20], [1000, 7]],
                         ids=["mma_sync_scan", "short_tc_and_persistent_scan", "short_rec", "only_short", "2seq"])
def test_prefill_in_place_state_dps(lens):
    """new_state may be the state tensor itself (in-place write-back) on every route: each CTA
    reads its slice of the initial state before it writes that slice."""
    inp = gi.prefill_inputs(lens, seed=26)
    args = util.prefill_args(inp)
    ro, rs = gdn.prefill.run(*args)
    q, k, v, st, A_log, a, dt_bias, b, cu, scale = args
    out = torch.empty_like(ro)
    gdn.prefill.kernel(q, k, v, st, A_log, a, dt_bias, b, cu, scale, out, st)
    torch.cuda.synchronize()
    assert torch.equal(out, ro) and torch.equal(st, rs)


def test_prefill_deterministic_and_bv_variants():
    from gdn import prefill as pmod

    inp = gi.prefill_inputs([300, 77], seed=27)
    args = util.prefill_args(inp)
    o1, s1 = gdn.prefill.run(*args)
    o2, s2 = gdn.prefill.run(*args)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    for bv in (16, 32):
        out = torch.empty_like(o1)
        ns = torch.empty_like(s1)
        pmod._launch(*args, out, ns, flags=bv << 8)
        torch.cuda.synchronize()
        assert torch.equal(out, o1) and torch.equal(ns, s1)


TC_CASES = [[300, 77], [1], [64], [130, 0, 77, 300], [1000], [6] * 40 + [100, 70]]


@pytest.mark.parametrize("lens", TC_CASES, ids=["300-77", "1", "64", "mixed4", "1000", "short42"])
@pytest.mark.parametrize("with_state", [True, False], ids=["h0", "zero"])
def test_prefill_tcgen05_scan_matches_oracle(lens, with_state):
    """The tcgen05 scan (64-column slices, the default for many sequences), forced on any batch."""
    from gdn import prefill as pmod

    inp = gi.prefill_inputs(lens, seed=40 + len(lens), with_state=with_state)
    args = util.prefill_args(inp)
    T, N = sum(lens), len(lens)
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(N, 8, 128, 128, dtype=torch.float32, device="cuda")
    pmod._launch(*args, out, ns, flags=64 << 8)
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


def test_prefill_strong_decay_extremes():
    inp = gi.prefill_inputs([130, 64], seed=28)
    inp["A_log"] = np.array([np.log(16.0), 0.0, -8.0, np.log(16.0), -20.0, 2.0, 0.5, -1.0], np.float32)
    rng = np.random.default_rng(5)
    inp["a"] = gi.to_bf16_bits((rng.standard_normal((194, 8)) * 10).astype(np.float32))
    _run_and_check(inp)


@pytest.mark.parametrize("lens", [[256, 100], [300] * 4 + [64], [6] * 40 + [100, 0]],
                         ids=["mma_sync_scan", "tcgen05_scan", "short_path_table"])
def test_prefill_graph_capture(lens):
    """Every launch sequence (table, short, prep, both scans) captures into a CUDA graph and
    replays to the eager result: nothing is read back to the host."""
    inp = gi.prefill_inputs(lens, seed=29)
    q, k, v, st, A_log, a, dt_bias, b, cu, scale = util.prefill_args(inp)
    ro, rs = gdn.prefill.run(q, k, v, st, A_log, a, dt_bias, b, cu, scale)
    out = torch.empty_like(ro)
    ns = torch.empty_like(rs)
    ws = torch.empty(gdn.prefill.workspace_bytes(len(lens), sum(lens)), dtype=torch.uint8, device="cuda")
    from gdn import prefill as pmod

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        pmod._launch(q, k, v, st, A_log, a, dt_bias, b, cu, scale, out, ns, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        pmod._launch(q, k, v, st, A_log, a, dt_bias, b, cu, scale, out, ns, workspace=ws)
    out.zero_()
    ns.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ro) and torch.equal(ns, rs)


# ---- benchmark configurations at full size ------------------------------------------------

def test_prefill_config2_t1024():
    inp = gi.prefill_inputs([1024], seed=0, with_state=False)
    _run_and_check(inp)


def test_prefill_config3_varlen_16_seqs():
    lens = gi.varlen_lengths(16, 6, 8192, 32768, seed=0)
    inp = gi.prefill_inputs(lens, seed=0, with_state=True)
    _run_and_check(inp)


def test_prefill_8k_single_sequence():
    inp = gi.prefill_inputs([8192], seed=0, with_state=True)
    _run_and_check(inp)


def test_prefill_packed_8x1024():
    inp = gi.prefill_inputs([1024] * 8, seed=1, with_state=True)
    _run_and_check(inp)


def test_prefill_many_sequences_chunk_table_path():
    """More than 32 sequences: slots come from the one-CTA chunk-table kernel instead of a
    per-warp lookup; includes zero-length and single-token sequences."""
    rng = np.random.default_rng(31)
    lens = rng.integers(0, 90, 300).tolist()
    lens[5] = 0
    lens[7] = 1
    inp = gi.prefill_inputs(lens, seed=31)
    _run_and_check(inp)


def test_prefill_more_sequences_than_one_table_tile():
    """1100 short sequences: the chunk-table kernel's prefix sum spans two 1024-thread tiles."""
    rng = np.random.default_rng(32)
    lens = rng.integers(0, 4, 1100).tolist()
    inp = gi.prefill_inputs(lens, seed=32)
    _run_and_check(inp)


@pytest.mark.timeout(120)
@pytest.mark.parametrize("scan", [0, 64], ids=["mma_sync_scan", "tcgen05_scan"])
def test_prefill_bounded_wait_reports_and_recovers(scan):
    """Failure detection without a GPU fault: with the test hook the scan's producer withholds a
    chunk's TMA copies, the math warps' bounded mbarrier wait expires, the kernel records status 1
    in the workspace and returns; the context stays usable and the next call is correct.  Both
    scan kernels (mma.sync and tcgen05) are exercised."""
    from gdn import prefill as pmod

    inp = gi.prefill_inputs([200], seed=33)
    args = util.prefill_args(inp)
    out = torch.empty(200, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(1, 8, 128, 128, dtype=torch.float32, device="cuda")
    ws = torch.empty(gdn.prefill.workspace_bytes(1, 200), dtype=torch.uint8, device="cuda")
    pmod._launch(*args, out, ns, workspace=ws, flags=1 | (scan << 8))  # GDN_FLAG_TEST_WITHHOLD_CHUNK
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 1  # GDN_DEVSTATUS_SCAN_TMA_TIMEOUT
    pmod._launch(*args, out, ns, workspace=ws)
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 0
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


@pytest.mark.parametrize("lens", [[6] * 40, [1, 2, 3, 32, 0, 33, 5, 4] * 6, [8, 9, 16, 17, 1, 2, 3, 4] * 6,
                                  [1, 24, 25, 3, 200, 0, 17] * 6, [24] * 33, list(range(33)) + [40, 64, 65]],
                         ids=["40x6", "rec_mixed", "rec_block_edges", "mixed", "33x24", "tc_0to32"])
def test_prefill_short_sequence_path(lens):
    """In batches of more than 32 sequences, sequences of up to 32 tokens take a short-sequence
    kernel (the token recurrence when the batch averages at most 10 tokens per sequence, the
    one-chunk tensor-core kernel otherwise) and longer ones the chunked kernels, in the same call;
    both must match the oracle, and the chunked-only route (GDN_FLAG_NO_SHORT_PATH) must agree."""
    from gdn import prefill as pmod

    inp = gi.prefill_inputs(lens, seed=34 + len(lens))
    _run_and_check(inp)
    args = util.prefill_args(inp)
    o1, s1 = gdn.prefill.run(*args)
    o2 = torch.empty_like(o1)
    s2 = torch.empty_like(s1)
    pmod._launch(*args, o2, s2, flags=2)  # GDN_FLAG_NO_SHORT_PATH
    torch.cuda.synchronize()
    util.check_out(util.bits(o2), util.bits(o1), atol=2e-3, rtol=2e-2)
    util.check_state(s2.cpu().numpy(), s1.cpu().numpy(), rel_l2=1e-4)


def test_prefill_persistent_grids_many_items():
    """With the short path on (more than 32 sequences), the prep and tcgen05-scan kernels run
    persistent grids of at most one or two CTAs per SM that take work items from device counters.
    160 sequences of 33-300 tokens plus short ones give ~2,500 scan items and ~2,800 prep items,
    so every CTA runs many items back to back (mbarrier phases carried across items).  The result
    must match the oracle and the one-CTA-per-item route (GDN_FLAG_NO_SHORT_PATH)."""
    from gdn import prefill as pmod

    rng = np.random.default_rng(41)
    lens = rng.integers(33, 301, 160).tolist() + [0, 5, 32, 1] * 5
    rng.shuffle(lens)
    inp = gi.prefill_inputs(lens, seed=41)
    _run_and_check(inp)
    args = util.prefill_args(inp)
    o1, s1 = gdn.prefill.run(*args)
    o2 = torch.empty_like(o1)
    s2 = torch.empty_like(s1)
    pmod._launch(*args, o2, s2, flags=2)  # GDN_FLAG_NO_SHORT_PATH
    torch.cuda.synchronize()
    util.check_out(util.bits(o2), util.bits(o1), atol=2e-3, rtol=2e-2)
    util.check_state(s2.cpu().numpy(), s1.cpu().numpy(), rel_l2=1e-4)


@pytest.mark.timeout(120)
def test_prefill_bounded_wait_persistent_scan():
    """Failure detection inside the persistent tcgen05 scan: with the test hook every item's
    second chunk is withheld, the bounded waits expire, each CTA records status 1, leaves its item
    loop and frees its TMEM; the next call on the same workspace is correct."""
    from gdn import prefill as pmod

    lens = [100] * 40
    inp = gi.prefill_inputs(lens, seed=42)
    args = util.prefill_args(inp)
    T = sum(lens)
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(len(lens), 8, 128, 128, dtype=torch.float32, device="cuda")
    ws = torch.empty(gdn.prefill.workspace_bytes(len(lens), T), dtype=torch.uint8, device="cuda")
    pmod._launch(*args, out, ns, workspace=ws, flags=1 | (64 << 8))  # GDN_FLAG_TEST_WITHHOLD_CHUNK
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 1  # GDN_DEVSTATUS_SCAN_TMA_TIMEOUT
    pmod._launch(*args, out, ns, workspace=ws)
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 0
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


@pytest.mark.parametrize("lens,cu", [([6], None), ([32], None), ([0, 5, 0, 12], None), ([16, 16], None),
                                     ([30], [3, 23]), ([9], [2, 7])],
                         ids=["1x6_rec", "1x32_tc", "4_seqs_rec", "2x16_tc", "unowned_tc", "unowned_rec"])
def test_prefill_only_short_single_launch(lens, cu):
    """T <= 32: every sequence is short, so the short-sequence kernel (the token recurrence when
    T <= 10 N, else the one-chunk tensor-core kernel) is the call's only launch and also zeroes
    the output rows outside [cu[0], cu[N]) and the status word.  Must match the oracle and the
    chunked route (GDN_FLAG_NO_SHORT_PATH)."""
    from gdn import prefill as pmod

    inp = gi.prefill_inputs(lens, seed=43 + sum(lens))
    if cu is not None:
        inp["cu_seqlens"] = np.array(cu, np.int32)
    T = int(sum(lens))
    args = util.prefill_args(inp)
    out = torch.full((T, 8, 128), 7.0, dtype=torch.bfloat16, device="cuda")  # stale values must be overwritten
    ns = torch.empty(len(inp["cu_seqlens"]) - 1, 8, 128, 128, dtype=torch.float32, device="cuda")
    ws = torch.empty(gdn.prefill.workspace_bytes(ns.shape[0], T), dtype=torch.uint8, device="cuda")
    ws.fill_(0xFF)  # stale status word
    pmod._launch(*args, out, ns, workspace=ws)
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 0
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)
    o2 = torch.empty_like(out)
    s2 = torch.empty_like(ns)
    pmod._launch(*args, o2, s2, flags=2)  # GDN_FLAG_NO_SHORT_PATH
    torch.cuda.synchronize()
    util.check_out(util.bits(o2), util.bits(out), atol=2e-3, rtol=2e-2)
    util.check_state(s2.cpu().numpy(), ns.cpu().numpy(), rel_l2=1e-4)


def _all_same_inputs(T):
    """The adversarial input noted for the reference's fast path (every tensor 0.5): with |k|^2 = 32
    the delta rule multiplies the state by ~-19 per token, so the sequential oracle reaches ~1e22
    at 64 tokens and overflows near 100."""
    half = np.uint16(0x3F00)  # 0.5 in bf16
    return dict(q=np.full((T, 4, 128), half), k=np.full((T, 4, 128), half), v=np.full((T, 8, 128), half),
                state=np.full((1, 8, 128, 128), 0.5, np.float32), A_log=np.full(8, 0.5, np.float32),
                a=np.full((T, 8), half), dt_bias=np.full(8, 0.5, np.float32), b=np.full((T, 8), half),
                cu_seqlens=np.array([0, T], np.int32), scale=0.5)


@pytest.mark.parametrize("T,flags", [(8, 0), (8, 2), (24, 0), (64, 0)],
                         ids=["8_recurrent", "8_chunked", "24_short_tc", "64_chunked"])
def test_prefill_all_same_input_stays_finite(T, flags):
    """Every route stays finite where the oracle does (the reference's chunked path returns NaN
    here).  The token recurrence matches at the usual bar; the chunked forms, whose inverse
    (I + A)^-1 has entries ~20^n on this input, stay within 1% of the output's scale and 1e-2 state
    rel-L2."""
    from gdn import prefill as pmod

    inp = _all_same_inputs(T)
    args = util.prefill_args(inp)
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(1, 8, 128, 128, dtype=torch.float32, device="cuda")
    pmod._launch(*args, out, ns, flags=flags)
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    got = util.bf16_bits_to_f32(util.bits(out)).astype(np.float64)
    ref = util.bf16_bits_to_f32(ro).astype(np.float64)
    st, rs64 = ns.cpu().numpy().astype(np.float64), rs.astype(np.float64)
    assert np.isfinite(got).all() and np.isfinite(st).all()
    rel_state = np.linalg.norm(st - rs64) / np.linalg.norm(rs64)
    if T == 8 and flags == 0:  # token-recurrent short kernel
        util.check_out(util.bits(out), ro)
        assert rel_state < util.STATE_REL_L2
    else:
        assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()
        assert rel_state < 1e-2


@pytest.mark.parametrize("scan", [16, 64], ids=["mma_sync_scan", "tcgen05_scan"])
def test_prefill_overlapping_cu_seqlens_stays_in_bounds(scan):
    """cu_seqlens that is not non-decreasing: sequence 3 = [128, 640) overlaps sequences 0 and 1, so
    the sequences claim 16 chunks where the workspace holds 14 slots.  The kernels skip the excess
    chunks, report GDN_DEVSTATUS_BAD_SEQLENS (5) and stay inside every buffer; sequence 0's slots
    come first, so its final state is still that of sequence 0 alone."""
    from gdn import prefill as pmod

    T = 640
    inp = gi.prefill_inputs([T], seed=35, with_state=True)
    inp["state"] = np.concatenate([inp["state"]] * 4)
    cu = torch.tensor([0, 256, 512, 128, 640], dtype=torch.int32, device="cuda")
    args = list(util.prefill_args(inp))
    args[8] = cu
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(4, 8, 128, 128, dtype=torch.float32, device="cuda")
    ws = torch.empty(gdn.prefill.workspace_bytes(4, T), dtype=torch.uint8, device="cuda")
    pmod._launch(*args, out, ns, workspace=ws, flags=scan << 8)
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 5
    one = dict(inp, state=inp["state"][:1], cu_seqlens=np.array([0, 256], np.int32))
    for key in ("q", "k", "v", "a", "b"):
        one[key] = inp[key][:256]
    _, rs = _oracle(one)
    util.check_state(ns[:1].cpu().numpy(), rs)
