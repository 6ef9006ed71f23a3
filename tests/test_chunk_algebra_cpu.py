"""CPU check of the chunked recurrence's precision, independent of the GPU.

The prefill kernels run the chunk-level WY form of the delta rule
(solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:858-905 for A,
197-314 for (I + A)^-1, 334-383 for w and u, 503-645 for the chunk recurrence) with bf16 tensor-core
operands.  This file emulates that recurrence in numpy, rounding to bf16 exactly where the kernels
do, and compares the final state with the sequential oracle (a C restatement of
reference/gdn_prefill_ref.py:42-91).  It checks two per-chunk forms of the state step:

* the form the kernels use: vn = (u - w h) e^{G_L - G}, split into bf16 hi + lo, then
  h' = e^{G_L} h + K^T vn;
* the transition form: h' = e^{G_L} h + K^T (d u) - M h with M = K^T diag(d) w rounded to bf16
  (d = e^{G_L - G}), so the dependent chain is one product per chunk.

Weak decay (A_log = -6) makes the state remember thousands of tokens, the hardest case for bf16
operands.  Both forms have to stay within the 3e-3 state rel-L2 that the GPU tests allow there,
and within 1e-4 on the benchmark's input distribution.
"""
import numpy as np
import pytest

from oracle import oracle
from tests.golden import inputs as gi

C = 64


def _rb(x):
    return gi.bf16_bits_to_f32(gi.to_bf16_bits(np.asarray(x, np.float32)))


def _chunked_state(inp, form, heads):
    q_h = inp["q"].shape[1]
    k = gi.bf16_bits_to_f32(inp["k"])
    v = gi.bf16_bits_to_f32(inp["v"])
    a = gi.bf16_bits_to_f32(inp["a"])
    b = gi.bf16_bits_to_f32(inp["b"])
    hv_n = v.shape[1]
    x = a + inp["dt_bias"][None, :]
    softplus = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))
    g = (-np.exp(inp["A_log"])[None, :] * softplus).astype(np.float32)
    beta = (1 / (1 + np.exp(-b))).astype(np.float32)
    T = k.shape[0]
    out = {}
    for hv in heads:
        kk = k[:, hv // (hv_n // q_h)]
        h = inp["state"][0, hv].T.astype(np.float32).copy()  # [K, V]
        for c0 in range(0, T, C):
            L = min(C, T - c0)
            kc, vc = kk[c0:c0 + L], v[c0:c0 + L, hv]
            gc, bc = g[c0:c0 + L, hv], beta[c0:c0 + L, hv]
            G = np.cumsum(gc).astype(np.float32)
            decay = np.exp(np.minimum(G[:, None] - G[None, :], 0))
            A = np.tril(bc[:, None] * decay * (kc @ kc.T), -1)
            Tm = np.linalg.inv(np.eye(L) + A).astype(np.float32)
            w = _rb(_rb(Tm) @ (bc[:, None] * np.exp(G)[:, None] * kc))
            u = (_rb(Tm - np.eye(L)) @ (bc[:, None] * vc) + bc[:, None] * vc).astype(np.float32)
            d = np.exp(G[-1] - G).astype(np.float32)
            eL = np.float32(np.exp(G[-1]))
            if form == "vn_split":
                vn = (u - w @ _rb(h)) * d[:, None]
                hi = _rb(vn)
                h = eL * h + kc.T @ (hi + _rb(vn - hi))
            else:
                du = d[:, None] * u
                hi = _rb(du)
                M = _rb(kc.T @ _rb(d[:, None] * w))
                h = eL * h + kc.T @ (hi + _rb(du - hi)) - M @ _rb(h)
        out[hv] = h.T
    return out


def _rel(a, b):
    return float(np.linalg.norm((a - b).astype(np.float64)) / np.linalg.norm(b.astype(np.float64)))


@pytest.mark.parametrize("form", ["vn_split", "transition"])
@pytest.mark.parametrize("case", ["benchmark", "weak_decay"])
def test_chunked_form_matches_sequential_oracle(form, case):
    inp = gi.prefill_inputs([1024], seed=78, with_state=True)
    bar = 1e-4
    if case == "weak_decay":
        inp["A_log"] = np.full(8, -6.0, np.float32)
        bar = 3e-3
    _, ref = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["cu_seqlens"], inp["scale"])
    heads = (0, 5)
    got = _chunked_state(inp, form, heads)
    for hv in heads:
        assert _rel(got[hv], ref[0, hv]) < bar
