"""The oracle's in-kernel L2-norm variant (q, k normalised per token and head before the step,
x * (sum x^2 + 1e-6)^-1/2 as in the reference's decode sweep kernel,
tests/bench_decode_sweep.py:43-46) against an independent float64 restatement of the
reference recurrence (reference/gdn_decode_ref.py:42-83, reference/gdn_prefill_ref.py:42-91)."""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import oracle
from tests.golden import inputs as gi

H, HV, D = 4, 8, 128


def _f64_step(S, q, k, v, g, beta, scale):
    """One token on a [K, V] float64 state, the reference's order of operations."""
    S = S * g
    old = k @ S
    new = beta * v + (1.0 - beta) * old
    S = S - np.outer(k, old) + np.outer(k, new)
    return S, scale * (q @ S)


def _gates(a, b, A_log, dt_bias):
    x = float(a) + float(dt_bias)
    sp = x if x > 20.0 else math.log1p(math.exp(x))
    return math.exp(-math.exp(float(A_log)) * sp), 1.0 / (1.0 + math.exp(-float(b)))


def _l2(x):
    return x / math.sqrt(float((x.astype(np.float64) ** 2).sum()) + 1e-6)


def _f64_prefill(inp):
    f = gi.bf16_bits_to_f32
    q, k, v, a, b = (f(inp[n]).astype(np.float64) for n in ("q", "k", "v", "a", "b"))
    cu = inp["cu_seqlens"]
    N = len(cu) - 1
    T = q.shape[0]
    out = np.zeros((T, HV, D))
    ns = np.zeros((N, HV, D, D))
    for n in range(N):
        for hv in range(HV):
            S = inp["state"][n, hv].astype(np.float64).T.copy()  # k-last [V, K] -> [K, V]
            for t in range(cu[n], cu[n + 1]):
                g, beta = _gates(a[t, hv], b[t, hv], inp["A_log"][hv], inp["dt_bias"][hv])
                S, o = _f64_step(S, _l2(q[t, hv // 2]), _l2(k[t, hv // 2]), v[t, hv], g, beta, inp["scale"])
                out[t, hv] = o
            if cu[n + 1] > cu[n]:
                ns[n, hv] = S.T
    return out, ns


@pytest.mark.parametrize("lens", [[1], [5, 9], [3, 0, 7]])
def test_oracle_l2norm_prefill_matches_float64(lens):
    inp = gi.prefill_inputs(lens, seed=71 + len(lens), normalized=False)
    out, ns = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                             inp["b"], inp["cu_seqlens"], inp["scale"], qk_l2norm=True)
    ro, rs = _f64_prefill(inp)
    np.testing.assert_allclose(gi.bf16_bits_to_f32(out), ro, atol=1e-2, rtol=1e-2)
    assert np.linalg.norm(ns - rs) <= 1e-5 * max(np.linalg.norm(rs), 1e-30)


def test_oracle_l2norm_decode_equals_prefill_t1():
    """Decode with the L2 norm equals a one-token prefill with it, bit for bit."""
    d = gi.decode_inputs(3, seed=5, normalized=False)
    o1, s1 = oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], d["scale"],
                           qk_l2norm=True)
    cu = np.arange(4, dtype=np.int64)
    o2, s2 = oracle.prefill(d["q"][:, 0], d["k"][:, 0], d["v"][:, 0], d["state"], d["A_log"], d["a"][:, 0],
                            d["dt_bias"], d["b"][:, 0], cu, d["scale"], qk_l2norm=True)
    assert np.array_equal(o1[:, 0], o2) and np.array_equal(s1, s2)


def test_oracle_l2norm_on_unit_norm_inputs_matches_official_oracle():
    """On inputs that are already unit-norm the variant is the official oracle up to rounding."""
    inp = gi.prefill_inputs([40], seed=9)
    args = (inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
            inp["cu_seqlens"], inp["scale"])
    o0, s0 = oracle.prefill(*args)
    o1, s1 = oracle.prefill(*args, qk_l2norm=True)
    np.testing.assert_allclose(gi.bf16_bits_to_f32(o1), gi.bf16_bits_to_f32(o0), atol=2e-2, rtol=2e-2)
    assert np.linalg.norm(s1 - s0) <= 1e-2 * np.linalg.norm(s0)
