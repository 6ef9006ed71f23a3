"""The segmented prefill route (csrc/prefill_seg.cu) against the CPU oracle and against the
single-pass scan.  One sequence of >= 3072 tokens, or a few averaging >= 6144, take it by default;
GDN_FLAG_SEGMENTS forces it for the other calls whose workspace has its regions,
GDN_FLAG_NO_SEGMENTS forces the single-pass scan, and bits 16-23 force a segment length.  Cases cover one sequence, several, ragged tails, a one-token and a
zero-length sequence, and segment lengths that do and do not divide the chunk count."""
import numpy as np
import pytest
import torch

import gdn
from gdn import prefill as pmod
from oracle import oracle
from tests import util
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

NO_SEGMENTS = 0x8
SEGMENTS = 0x10


def _call(inp, flags=0):
    args = util.prefill_args(inp)
    T = args[0].shape[0]
    N = args[8].shape[0] - 1
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(N, 8, 128, 128, dtype=torch.float32, device="cuda")
    ws = torch.empty(gdn.prefill.workspace_bytes(N, T), dtype=torch.uint8, device="cuda")
    pmod._launch(*args, out, ns, workspace=ws, flags=flags)
    torch.cuda.synchronize()
    assert gdn.prefill.read_status(ws) == 0
    return out, ns


def _oracle(inp):
    return oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                          inp["b"], inp["cu_seqlens"], inp["scale"])


CASES = [
    ([8192], True), ([4096], False), ([1024], True), ([600], True), ([777], True),
    ([3000, 2000], True), ([1000, 1, 700], True), ([600, 0, 1000], True), ([513, 1100, 64, 900], True),
]


@pytest.mark.parametrize("lens,with_state", CASES, ids=["-".join(map(str, l)) for l, _ in CASES])
def test_segmented_prefill_matches_oracle(lens, with_state):
    inp = gi.prefill_inputs(lens, seed=1000 + sum(lens), with_state=with_state)
    out, ns = _call(inp, SEGMENTS)
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)
    # the single-pass scan on the same inputs agrees to the parity bar as well
    out1, ns1 = _call(inp, NO_SEGMENTS)
    util.check_out(util.bits(out), util.bits(out1))
    util.check_state(ns.cpu().numpy(), ns1.cpu().numpy())


@pytest.mark.parametrize("m", [8, 11, 31, 64, 128])
def test_segmented_prefill_forced_segment_lengths(m):
    """Segment lengths from the default (8 chunks at 4096 tokens) up to the whole sequence (one
    segment) give the oracle's results.  Shorter ones would need more segment slots than the
    workspace holds (GDN_ERR_SIZE, checked below)."""
    inp = gi.prefill_inputs([4096], seed=77, with_state=True)
    out, ns = _call(inp, SEGMENTS | (m << 16))
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


def test_segmented_prefill_weak_decay_long_memory():
    """Weak decay (A_log = -6: the state remembers thousands of tokens) is the hard case for the
    segment transitions, which then carry most of the state across segments."""
    inp = gi.prefill_inputs([4096], seed=78, with_state=True)
    inp["A_log"] = np.full(8, -6.0, np.float32)
    out, ns = _call(inp, SEGMENTS)
    out1, ns1 = _call(inp, NO_SEGMENTS)
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    # both routes round W, h and X to bf16 as MMA operands; at this memory length that costs
    # about 1e-3 of state rel-L2 for either route (measured in a numpy emulation)
    rel = util.check_state(ns.cpu().numpy(), rs, rel_l2=3e-3)
    rel1 = util.check_state(ns1.cpu().numpy(), rs, rel_l2=3e-3)
    assert rel <= 2 * rel1 + 1e-4


def test_segmented_prefill_in_place_and_graph_capture():
    """new_state aliasing state (destination-passing, in place) and replay from a CUDA graph, on
    the default route of two long sequences (segmented)."""
    inp = gi.prefill_inputs([6400, 7000], seed=79, with_state=True)
    ro, rs = _oracle(inp)
    args = list(util.prefill_args(inp))
    st = args[3]
    out = torch.empty(13400, 8, 128, dtype=torch.bfloat16, device="cuda")
    g = torch.cuda.CUDAGraph()
    s0 = st.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        gdn.prefill.kernel(*args[:3], st, *args[4:], out, st)  # warm-up (also the first in-place call)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    util.check_out(util.bits(out), ro)
    util.check_state(st.cpu().numpy(), rs)
    st.copy_(s0)
    with torch.cuda.graph(g):
        gdn.prefill.kernel(*args[:3], st, *args[4:], out, st)
    out.zero_()
    st.copy_(s0)
    g.replay()
    torch.cuda.synchronize()
    util.check_out(util.bits(out), ro)
    util.check_state(st.cpu().numpy(), rs)


def test_segmented_prefill_rejects_segments_beyond_the_workspace():
    inp = gi.prefill_inputs([4096], seed=80, with_state=True)
    with pytest.raises(gdn.GDNError) as e:
        _call(inp, SEGMENTS | (2 << 16))
    assert e.value.status == 4  # GDN_ERR_SIZE


def test_segmented_route_is_the_default_for_long_sequences():
    """Default flags on a 1 x 8192 call give the same bits as forcing the segmented route."""
    inp = gi.prefill_inputs([8192], seed=81, with_state=True)
    o1, s1 = _call(inp)
    o2, s2 = _call(inp, SEGMENTS)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert torch.equal(s1.view(torch.int32), s2.view(torch.int32))


@pytest.mark.parametrize("h,hv", [(1, 2), (1, 1), (2, 4)], ids=["qk1_v2", "qk1_v1", "qk2_v4"])
@pytest.mark.parametrize("lens", [[3000, 700, 64, 1], [6500]], ids=["mixed4", "6500"])
def test_segmented_prefill_few_v_heads(h, hv, lens):
    """The segmented route with the few v-heads of one head-split piece (its segment length then comes
    from the lower bound m^2 >= chunks / 3) and the single-pass scan on the same inputs, both against the
    oracle, for several sequences and for one long one."""
    inp = gi.prefill_inputs(lens, seed=1300 + h + hv + len(lens), h=h, hv=hv)
    args = util.prefill_args(inp)
    T, N = args[0].shape[0], args[8].shape[0] - 1
    outs = []
    for flags in (SEGMENTS, NO_SEGMENTS):
        out = torch.empty(T, hv, 128, dtype=torch.bfloat16, device="cuda")
        ns = torch.empty(N, hv, 128, 128, dtype=torch.float32, device="cuda")
        ws = torch.empty(gdn.prefill.workspace_bytes(N, T, h, hv), dtype=torch.uint8, device="cuda")
        pmod._launch(*args, out, ns, workspace=ws, flags=flags)
        torch.cuda.synchronize()
        assert gdn.prefill.read_status(ws) == 0
        outs.append((out, ns))
    ro, rs = _oracle(inp)
    for out, ns in outs:
        util.check_out(util.bits(out), ro)
        util.check_state(ns.cpu().numpy(), rs)
