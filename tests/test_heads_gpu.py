"""Other head-count families on the GPU (a superset of the reference, which fixes 4 q/k heads and
8 v-heads): H q/k heads and HV v-heads with HV a multiple of H, v-head hv reading q/k head
hv // (HV // H).  Decode and prefill through the C ABI against the CPU oracle,
which takes the head counts from the input shapes.  qk16_v32 is the family of the contest
workloads the reference was written for."""
import pytest
import torch

import gdn
from oracle import oracle
from tests import util
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

DECODE_FAMILIES = [(16, 32), (8, 16), (2, 8), (8, 8), (4, 12), (1, 2)]


@pytest.mark.parametrize("h,hv", DECODE_FAMILIES, ids=[f"qk{h}_v{v}" for h, v in DECODE_FAMILIES])
@pytest.mark.parametrize("B", [1, 33])
def test_decode_head_families_match_oracle(h, hv, B):
    inp = gi.decode_inputs(B, seed=500 + h * 7 + hv + B, h=h, hv=hv)
    out, ns = gdn.decode.run(*util.decode_args(inp))
    torch.cuda.synchronize()
    ro, rs = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                           inp["b"], inp["scale"])
    assert out.shape == (B, 1, hv, 128)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs, rel_l2=1e-5)


PREFILL_FAMILIES = [(16, 32), (8, 16), (2, 8), (8, 8), (4, 16), (4, 12), (2, 4), (1, 2), (1, 1)]
PREFILL_LENS = [[200], [64, 1, 0, 130], [6] * 36 + [90], [20] * 36 + [90], [5, 9, 0, 12], [20]]


@pytest.mark.parametrize("h,hv", PREFILL_FAMILIES, ids=[f"qk{h}_v{v}" for h, v in PREFILL_FAMILIES])
@pytest.mark.parametrize("lens", PREFILL_LENS, ids=["200", "mixed4", "short37", "short37tc", "only_short_rec", "only_short_tc"])
def test_prefill_head_families_match_oracle(h, hv, lens):
    inp = gi.prefill_inputs(lens, seed=600 + h + hv + len(lens), h=h, hv=hv)
    out, ns = gdn.prefill.run(*util.prefill_args(inp))
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"])
    assert out.shape == (sum(lens), hv, 128)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


def test_prefill_qk16_v32_long_with_l2norm():
    """qk16_v32 with a 1100-token sequence and the in-kernel L2 norm."""
    inp = gi.prefill_inputs([1100, 300], seed=77, h=16, hv=32, normalized=False)
    out, ns = gdn.prefill.run(*util.prefill_args(inp), use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"], qk_l2norm=True)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("lens", [[8192], [3000, 64, 1000]], ids=["8192", "mixed3"])
def test_prefill_head_split_of_reference_family(world, lens):
    """One call of the reference family (4 q/k heads, 8 v-heads) run as `world` calls, each on one
    head_shard group (2 + 4, 1 + 2 or 1 + 1 heads: gates read with plain loads, and for 8192 tokens
    the segmented route with a segment length chosen for few v-heads), as ranks of a multi-GPU
    split would; the pieces put together match the oracle of the whole call."""
    from gdn.shard import head_shard

    inp = gi.prefill_inputs(lens, seed=900 + world + len(lens))
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"])
    outs, states = [], []
    for r in range(world):
        h0, h1, v0, v1 = head_shard(4, 8, world, r, prefill=True)
        part = dict(inp, q=inp["q"][:, h0:h1], k=inp["k"][:, h0:h1], v=inp["v"][:, v0:v1], state=inp["state"][:, v0:v1],
                    A_log=inp["A_log"][v0:v1], a=inp["a"][:, v0:v1], dt_bias=inp["dt_bias"][v0:v1], b=inp["b"][:, v0:v1])
        o, ns = gdn.prefill.run(*util.prefill_args(part))
        outs.append(util.bits(o))
        states.append(ns.cpu().numpy())
    torch.cuda.synchronize()
    import numpy as np
    util.check_out(np.concatenate(outs, axis=1), ro)
    util.check_state(np.concatenate(states, axis=1), rs)


def test_prefill_head_split_l2norm_int64_cu():
    """The 4-way head split pieces (1 q/k head, 2 v-heads each) with the in-kernel L2 norm and int64 cu_seqlens,
    on a batch of mixed lengths (6144 tokens down to 1)."""
    from gdn.shard import head_shard

    inp = gi.prefill_inputs([6144, 40, 1, 700], seed=931, normalized=False)
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"], qk_l2norm=True)
    import numpy as np
    outs, states = [], []
    for r in range(4):
        h0, h1, v0, v1 = head_shard(4, 8, 4, r, prefill=True)
        part = dict(inp, q=inp["q"][:, h0:h1], k=inp["k"][:, h0:h1], v=inp["v"][:, v0:v1], state=inp["state"][:, v0:v1],
                    A_log=inp["A_log"][v0:v1], a=inp["a"][:, v0:v1], dt_bias=inp["dt_bias"][v0:v1], b=inp["b"][:, v0:v1])
        o, ns = gdn.prefill.run(*util.prefill_args(part, cu_dtype=torch.int64), use_qk_l2norm_in_kernel=True)
        outs.append(util.bits(o))
        states.append(ns.cpu().numpy())
    torch.cuda.synchronize()
    util.check_out(np.concatenate(outs, axis=1), ro)
    util.check_state(np.concatenate(states, axis=1), rs)
