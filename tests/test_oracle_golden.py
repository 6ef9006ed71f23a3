"""Pin the CPU oracle (oracle/gdn_oracle.c) to the reference's own outputs.

The fixtures under tests/golden were produced by running the reference's
PyTorch oracles (reference/gdn_decode_ref.py::run, reference/gdn_prefill_ref.py::run)
on seeded inputs; the oracle must reproduce them to fp32 round-off.
"""
import numpy as np
import pytest

from oracle import oracle
from tests.golden import check, inputs as gi

DECODE = check.fixtures("decode")
PREFILL = check.fixtures("prefill")


@pytest.mark.parametrize("name,fx", DECODE, ids=[n for n, _ in DECODE])
def test_decode_oracle_matches_reference(name, fx):
    inp = check.regen(fx)
    out, ns = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                            inp["b"], inp["scale"])
    # bf16 output: allow one bf16 ulp of re-rounding; fp32 state: round-off only.
    check.compare(fx, "out", out, atol=1e-5, rtol=8e-3, proj_rtol=1e-3)
    check.compare(fx, "state", ns, atol=1e-6, rtol=1e-5, proj_rtol=1e-5)


@pytest.mark.parametrize("name,fx", PREFILL, ids=[n for n, _ in PREFILL])
def test_prefill_oracle_matches_reference(name, fx):
    inp = check.regen(fx)
    out, ns = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"],
                             inp["b"], inp["cu_seqlens"], inp["scale"])
    check.compare(fx, "out", out, atol=1e-5, rtol=8e-3, proj_rtol=1e-3)
    check.compare(fx, "state", ns, atol=1e-6, rtol=1e-5, proj_rtol=1e-5)


def test_prefill_t1_equals_decode():
    """A one-token prefill is one decode step (the reference oracles agree bit for bit)."""
    d = gi.decode_inputs(B=2, seed=5)
    T = 2
    q = d["q"].reshape(T, 4, 128)
    k = d["k"].reshape(T, 4, 128)
    v = d["v"].reshape(T, 8, 128)
    a = d["a"].reshape(T, 8)
    b = d["b"].reshape(T, 8)
    cu = np.array([0, 1, 2], np.int32)
    o1, s1 = oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], d["scale"])
    o2, s2 = oracle.prefill(q, k, v, d["state"], d["A_log"], a, d["dt_bias"], b, cu, d["scale"])
    assert np.array_equal(o1.reshape(-1), o2.reshape(-1))
    assert np.array_equal(s1, s2)


def test_oracle_thread_count_invariant():
    inp = gi.prefill_inputs([40, 23], seed=3)
    args = (inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
            inp["cu_seqlens"], inp["scale"])
    o1, s1 = oracle.prefill(*args, threads=1)
    o2, s2 = oracle.prefill(*args, threads=4)
    assert np.array_equal(o1, o2) and np.array_equal(s1, s2)


def test_scale_default():
    """scale None or 0 means 1/sqrt(128) (reference/gdn_decode_ref.py:38-39)."""
    d = gi.decode_inputs(B=1, seed=6)
    args = [d[x] for x in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")]
    o0, _ = oracle.decode(*args, 0.0)
    on, _ = oracle.decode(*args, None)
    os_, _ = oracle.decode(*args, 1.0 / np.sqrt(128.0))
    assert np.array_equal(o0, os_) and np.array_equal(on, os_)
