"""Full-size prefill checks: the BASELINE multi-GPU configuration (64 x 4096 tokens) against the
CPU oracle, and size-independent properties at the benchmark's sizes: a sequence split at a chunk boundary and continued from the carried
state gives the same outputs and final state as one call (the recurrence is the same one,
reference/gdn_prefill_ref.py:56-89), and a packed batch gives, for every sequence, what the
sequence gives alone (sequences are independent, reference/gdn_prefill_ref.py:56).  Inputs are
generated on the GPU with the benchmark's distributions."""
import pytest
import torch

import gdn
from tests import util

pytestmark = pytest.mark.gpu


def _inputs(lens, seed, H=4, HV=8):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T, N = sum(lens), len(lens)
    rn = lambda *s: torch.randn(*s, generator=g, device="cuda")
    l2n = lambda x: (x / x.norm(dim=-1, keepdim=True)).bfloat16()
    cu = torch.zeros(N + 1, dtype=torch.int32, device="cuda")
    cu[1:] = torch.tensor(lens, device="cuda").cumsum(0)
    return dict(q=l2n(rn(T, H, 128)), k=l2n(rn(T, H, 128)), v=rn(T, HV, 128).bfloat16(), state=rn(N, HV, 128, 128) * 0.02,
                A_log=torch.rand(HV, generator=g, device="cuda") * 2.7726, a=rn(T, HV).bfloat16(), dt_bias=rn(HV) * 0.1,
                b=rn(T, HV).bfloat16(), cu=cu, scale=128 ** -0.5)


def _run(d, sl=slice(None), state=None, cu=None):
    return gdn.prefill.run(d["q"][sl], d["k"][sl], d["v"][sl], d["state"] if state is None else state, d["A_log"],
                           d["a"][sl], d["dt_bias"], d["b"][sl], d["cu"] if cu is None else cu, d["scale"])


def _close(got, ref, atol=2e-3, rtol=2e-2, rel_l2=1e-4):
    if got.dtype == torch.bfloat16:
        util.check_out(util.bits(got), util.bits(ref), atol=atol, rtol=rtol)
    else:
        util.check_state(got.cpu().numpy(), ref.cpu().numpy(), rel_l2=rel_l2)


def test_prefill_8k_split_and_carry():
    """8192 tokens in one call == 4096 + 4096 with the state carried (mma.sync scan path)."""
    d = _inputs([8192], seed=1)
    o, s = _run(d)
    h = 4096
    cu = torch.tensor([0, h], dtype=torch.int32, device="cuda")
    o1, s1 = _run(d, slice(0, h), cu=cu)
    o2, s2 = _run(d, slice(h, 2 * h), state=s1, cu=cu)
    torch.cuda.synchronize()
    _close(torch.cat([o1, o2]), o)
    _close(s2, s)


def test_prefill_config4_split_and_carry_64x4096():
    """64 x 4096 tokens (the multi-GPU configuration at one GPU, tcgen05 scan path) == each
    sequence's first and second halves in two calls with the states carried."""
    L, N = 4096, 64
    d = _inputs([L] * N, seed=2)
    o, s = _run(d)
    half = L // 2
    idx1 = torch.cat([torch.arange(n * L, n * L + half, device="cuda") for n in range(N)])
    idx2 = idx1 + half
    cu = torch.arange(N + 1, dtype=torch.int32, device="cuda") * half
    sub = lambda idx: {**d, "q": d["q"][idx], "k": d["k"][idx], "v": d["v"][idx], "a": d["a"][idx], "b": d["b"][idx]}
    o1, s1 = _run(sub(idx1), cu=cu)
    o2, s2 = _run(sub(idx2), state=s1, cu=cu)
    torch.cuda.synchronize()
    got = torch.empty_like(o)
    got[idx1] = o1
    got[idx2] = o2
    _close(got, o)
    _close(s2, s)


def test_prefill_packing_invariance_config3():
    """The 16-sequence varlen batch packed in one call == each sequence alone (packed: tcgen05
    scan; alone: mma.sync scan)."""
    from tests.golden import inputs as gi

    lens = gi.varlen_lengths(16, 6, 8192, 32768, seed=0)
    d = _inputs(lens, seed=3)
    o, s = _run(d)
    starts = [0]
    for x in lens:
        starts.append(starts[-1] + x)
    for n, x in enumerate(lens):
        sl = slice(starts[n], starts[n + 1])
        cu = torch.tensor([0, x], dtype=torch.int32, device="cuda")
        on, sn = gdn.prefill.run(d["q"][sl], d["k"][sl], d["v"][sl], d["state"][n:n + 1], d["A_log"], d["a"][sl],
                                 d["dt_bias"], d["b"][sl], cu, d["scale"])
        torch.cuda.synchronize()
        _close(on, o[sl])
        _close(sn, s[n:n + 1])


def test_prefill_config4_64x4096_matches_oracle():
    """BASELINE config 4 at one GPU (64 sequences x 4096 tokens, per-sequence N(0, 0.02) initial
    state; the persistent tcgen05 scan route) against the CPU oracle, at the path's bar: output
    atol = rtol = 1e-2, final state rel-L2 1e-3.  The C oracle runs the 512 independent
    (sequence, v-head) recurrences on all host cores in a few seconds."""
    from oracle import oracle
    from tests.golden import inputs as gi

    inp = gi.prefill_inputs([4096] * 64, seed=64, with_state=True)
    out, ns = gdn.prefill.run(*util.prefill_args(inp))
    torch.cuda.synchronize()
    ro, rs = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"])
    util.check_out(util.bits(out), ro)
    util.check_state(ns.cpu().numpy(), rs)
