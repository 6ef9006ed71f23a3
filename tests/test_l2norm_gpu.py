"""In-kernel q/k L2-norm variant (GDN_FLAG_QK_L2NORM, ``use_qk_l2norm_in_kernel=True``) on the GPU:
decode and prefill on raw, un-normalised q / k against the CPU oracle with the same variant
(x * (sum x^2 + 1e-6)^-1/2 per token and head, tests/bench_decode_sweep.py:43-46), through the
C ABI.  The prefill cases cover one chunk, ragged multi-chunk sequences, zero-length sequences,
the short-sequence path (more than 32 sequences) and both scan slice widths."""
import numpy as np
import pytest
import torch

import gdn
from oracle import oracle
from tests import util
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B", [1, 8, 64])
def test_decode_l2norm_matches_oracle(B):
    inp = gi.decode_inputs(B, seed=300 + B, normalized=False)
    out, ns = gdn.decode.run(*util.decode_args(inp), use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    ro, rs = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                           inp["b"], inp["scale"], qk_l2norm=True)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs, rel_l2=1e-5)


def test_decode_l2norm_in_place_dps():
    inp = gi.decode_inputs(16, seed=9, normalized=False)
    args = util.decode_args(inp)
    st = args[3].clone()
    out = torch.empty(16, 1, 8, 128, dtype=torch.bfloat16, device="cuda")
    gdn.decode.kernel(*args[:3], st, *args[4:], out, st, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    ro, rs = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                           inp["b"], inp["scale"], qk_l2norm=True)
    util.check_out(util.bits(out), ro)
    util.check_state(st.cpu().numpy(), rs, rel_l2=1e-5)


PREFILL_CASES = [[1], [64], [200], [130, 0, 77, 300], [1024], [6] * 40 + [100, 3, 70], [20] * 40 + [100, 3, 70], [24]]


@pytest.mark.parametrize("lens", PREFILL_CASES, ids=["1", "64", "200", "mixed4", "1024", "short43", "short43tc", "only_short_tc"])
def test_prefill_l2norm_matches_oracle(lens):
    inp = gi.prefill_inputs(lens, seed=400 + len(lens), normalized=False)
    out, ns = gdn.prefill.run(*util.prefill_args(inp), use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"], qk_l2norm=True)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


def test_prefill_l2norm_on_unit_inputs_matches_plain_path():
    """On inputs that are already unit-norm the variant agrees with the default path."""
    inp = gi.prefill_inputs([300, 64], seed=12)
    args = util.prefill_args(inp)
    o0, s0 = gdn.prefill.run(*args)
    o1, s1 = gdn.prefill.run(*args, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    util.check_out(util.bits(o1), util.bits(o0))
    util.check_state(s1.cpu().numpy(), s0.cpu().numpy(), rel_l2=1e-3)
