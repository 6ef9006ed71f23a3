"""The oracle with other head-count families (H q/k heads, HV v-heads, HV a multiple of H) against
an independent float64 restatement of the reference recurrence (reference/gdn_prefill_ref.py:42-91,
GVA as repeat_interleave: v-head hv reads q/k head hv // (HV // H)), and the 4 / 8 family through
the same code path equal to the fixed-shape call."""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import oracle
from tests.golden import inputs as gi


def _gates(a, b, A_log, dt_bias):
    x = float(a) + float(dt_bias)
    sp = x if x > 20.0 else math.log1p(math.exp(x))
    return math.exp(-math.exp(float(A_log)) * sp), 1.0 / (1.0 + math.exp(-float(b)))


def _f64_prefill(inp):
    f = gi.bf16_bits_to_f32
    q, k, v, a, b = (f(inp[n]).astype(np.float64) for n in ("q", "k", "v", "a", "b"))
    H, HV, D = q.shape[1], v.shape[1], v.shape[2]
    cu = inp["cu_seqlens"]
    N = len(cu) - 1
    out = np.zeros((q.shape[0], HV, D))
    ns = np.zeros((N, HV, D, D))
    for n in range(N):
        for hv in range(HV):
            hq = hv // (HV // H)
            S = inp["state"][n, hv].astype(np.float64).T.copy()
            for t in range(cu[n], cu[n + 1]):
                g, beta = _gates(a[t, hv], b[t, hv], inp["A_log"][hv], inp["dt_bias"][hv])
                S = S * g
                old = k[t, hq] @ S
                new = beta * v[t, hv] + (1.0 - beta) * old
                S = S - np.outer(k[t, hq], old) + np.outer(k[t, hq], new)
                out[t, hv] = inp["scale"] * (q[t, hq] @ S)
            if cu[n + 1] > cu[n]:
                ns[n, hv] = S.T
    return out, ns


@pytest.mark.parametrize("h,hv", [(2, 4), (1, 3), (3, 3)])
def test_oracle_other_head_counts_match_float64(h, hv):
    inp = gi.prefill_inputs([4, 7], seed=20 + h + hv, h=h, hv=hv)
    out, ns = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                             inp["b"], inp["cu_seqlens"], inp["scale"])
    ro, rs = _f64_prefill(inp)
    assert out.shape == (11, hv, 128) and ns.shape == (2, hv, 128, 128)
    np.testing.assert_allclose(gi.bf16_bits_to_f32(out), ro, atol=1e-2, rtol=1e-2)
    assert np.linalg.norm(ns - rs) <= 1e-5 * np.linalg.norm(rs)


def test_oracle_decode_other_heads_equals_prefill_t1():
    d = gi.decode_inputs(2, seed=3, h=8, hv=16)
    o1, s1 = oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], d["scale"])
    cu = np.arange(3, dtype=np.int64)
    o2, s2 = oracle.prefill(d["q"][:, 0], d["k"][:, 0], d["v"][:, 0], d["state"], d["A_log"], d["a"][:, 0],
                            d["dt_bias"], d["b"][:, 0], cu, d["scale"])
    assert o1.shape == (2, 1, 16, 128)
    assert np.array_equal(o1[:, 0], o2) and np.array_equal(s1, s2)
