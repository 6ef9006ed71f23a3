"""Decode parity on the GPU: the CUDA path (through the C ABI) against the CPU oracle
and the reference's golden outputs, on the same seeded inputs."""
import numpy as np
import pytest
import torch

import gdn
from oracle import oracle
from tests import util
from tests.golden import check, inputs as gi

pytestmark = pytest.mark.gpu


def _oracle(inp):
    return oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                         inp["b"], inp["scale"])


@pytest.mark.parametrize("B", [1, 4, 8, 16, 32, 48, 64, 512])
def test_decode_matches_oracle(B):
    inp = gi.decode_inputs(B, seed=100 + B)
    out, ns = gdn.decode.run(*util.decode_args(inp))
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    assert out.shape == (B, 1, 8, 128) and ns.shape == (B, 8, 128, 128)
    util.check_out(util.bits(out), ro)
    rel = util.check_state(ns.cpu().numpy(), rs)
    # decode is fp32 end to end: far inside the 1e-3 bar
    assert rel < 1e-5


@pytest.mark.parametrize("name,fx", check.fixtures("decode"), ids=[n for n, _ in check.fixtures("decode")])
def test_decode_matches_reference_golden(name, fx):
    inp = check.regen(fx)
    out, ns = gdn.decode.run(*util.decode_args(inp))
    torch.cuda.synchronize()
    check.compare(fx, "out", util.bits(out), atol=util.OUT_ATOL, rtol=util.OUT_RTOL, proj_rtol=1e-2)
    check.compare(fx, "state", ns.cpu().numpy(), atol=1e-5, rtol=1e-4, proj_rtol=1e-4)


def test_decode_none_state_is_zero_state():
    inp = gi.decode_inputs(3, seed=7, with_state=False)
    out, ns = gdn.decode.run(*util.decode_args(inp))
    inp0 = dict(inp, state=np.zeros((3, 8, 128, 128), np.float32))
    out0, ns0 = gdn.decode.run(*util.decode_args(inp0))
    torch.cuda.synchronize()
    assert torch.equal(out, out0) and torch.equal(ns, ns0)
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


def test_decode_in_place_state_dps():
    """new_state may be the state tensor itself (in-place write-back)."""
    inp = gi.decode_inputs(16, seed=8)
    args = util.decode_args(inp)
    q, k, v, st, A_log, a, dt_bias, b, scale = args
    ref_out, ref_state = gdn.decode.run(*args)
    out = torch.empty(16, 1, 8, 128, dtype=torch.bfloat16, device="cuda")
    gdn.decode.kernel(q, k, v, st, A_log, a, dt_bias, b, scale, out, st)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert torch.equal(st, ref_state)


def test_decode_deterministic_and_scale_forms():
    inp = gi.decode_inputs(8, seed=9)
    args = list(util.decode_args(inp))
    o1, s1 = gdn.decode.run(*args)
    o2, s2 = gdn.decode.run(*args)
    args[-1] = torch.tensor(inp["scale"], device="cuda")
    o3, s3 = gdn.decode.run(*args)
    args[-1] = None
    o4, _ = gdn.decode.run(*args)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    assert torch.equal(o1, o3) and torch.equal(s1, s3)
    assert torch.equal(o1, o4)


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4])
def test_decode_all_tiling_variants(variant):
    """Every CTA tiling of the decode kernel gives the same bits."""
    from gdn import decode as dmod

    inp = gi.decode_inputs(24, seed=10)
    q, k, v, st, A_log, a, dt_bias, b, scale = util.decode_args(inp)
    ref_o, ref_s = gdn.decode.run(q, k, v, st, A_log, a, dt_bias, b, scale)
    out = torch.empty_like(ref_o)
    ns = torch.empty_like(ref_s)
    dmod._launch(q, k, v, st, A_log, a, dt_bias, b, scale, out, ns, flags=(variant + 1) << 8)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o) and torch.equal(ns, ref_s)


def test_decode_strong_and_weak_decay_extremes():
    inp = gi.decode_inputs(4, seed=11)
    inp["A_log"] = np.array([np.log(16.0), 0.0, -8.0, np.log(16.0), -20.0, 2.0, 0.5, -1.0], np.float32)
    inp["a"] = gi.to_bf16_bits(np.array([[[30.0, -30.0, 0.0, 5.0, -5.0, 25.0, 10.0, -10.0]]] * 4, np.float32))
    out, ns = gdn.decode.run(*util.decode_args(inp))
    torch.cuda.synchronize()
    ro, rs = _oracle(inp)
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)


def test_decode_graph_capture():
    inp = gi.decode_inputs(64, seed=12)
    q, k, v, st, A_log, a, dt_bias, b, scale = util.decode_args(inp)
    out = torch.empty(64, 1, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(st)
    ref_o, ref_s = gdn.decode.run(q, k, v, st, A_log, a, dt_bias, b, scale)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gdn.decode.kernel(q, k, v, st, A_log, a, dt_bias, b, scale, out, ns)  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gdn.decode.kernel(q, k, v, st, A_log, a, dt_bias, b, scale, out, ns)
    out.zero_()
    ns.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o) and torch.equal(ns, ref_s)
