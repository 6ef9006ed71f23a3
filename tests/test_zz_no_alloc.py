"""The allocation-free prefill entry point, gdn_prefill_fwd_noalloc.

Some callers cannot allocate device memory (a host runtime that owns all device
memory and forbids its plugins to call cudaMalloc, or a serving loop whose memory
is fixed at start-up).  gdn_prefill_fwd_noalloc serves them from a fixed scratch
array inside the library.  This test calls it through the C ABI and checks its
results against the regular entry point, gdn_prefill_fwd, on two calls in a row,
so contents left in the shared scratch array by the first call cannot leak into
the second.  The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from gdn import _lib
from tests import util
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu

MAX_TOKENS = 2048  # GDN_NOALLOC_MAX_TOKENS in include/gdn_b200.h
MAX_SEQS = 16      # GDN_NOALLOC_MAX_SEQS


def _noalloc_fn():
    lib = _lib.load()
    fn = lib.gdn_prefill_fwd_noalloc
    P, I, F, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_uint
    fn.argtypes = [P, P, P, P, P, P, P, P, P, I, I, I, F, P, P, I, I, I, I, P, U]
    fn.restype = I
    return fn


def _call_noalloc(fn, args, out, ns):
    q, k, v, st, A_log, a, dt_bias, b, cu, scale = args
    T = q.shape[0]
    N = cu.shape[0] - 1
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), None if st is None else st.data_ptr(), A_log.data_ptr(),
              a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(), 1 if cu.dtype == torch.int64 else 0,
              N, T, float(scale), out.data_ptr(), ns.data_ptr(), 4, 8, 128, 128, stream, 0)


def _call_regular(args, out, ns):
    q, k, v, st, A_log, a, dt_bias, b, cu, scale = args
    T = q.shape[0]
    N = cu.shape[0] - 1
    lib = _lib.load()
    need = lib.gdn_prefill_workspace_bytes(N, T, 4, 8, 128, 128)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    rc = lib.gdn_prefill_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), None if st is None else st.data_ptr(),
                             A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
                             1 if cu.dtype == torch.int64 else 0, N, T, float(scale), out.data_ptr(), ns.data_ptr(),
                             ws.data_ptr(), need, 4, 8, 128, 128, torch.cuda.current_stream().cuda_stream, 0)
    _lib.check("gdn_prefill_fwd", rc)
    torch.cuda.synchronize()
    return ws


def test_noalloc_prefill_matches_regular_entry_point_twice():
    fn = _noalloc_fn()
    cases = [
        gi.prefill_inputs([700, 64, 1, 300], seed=41, with_state=True),   # 1065 tokens, ragged tails
        gi.prefill_inputs([2000, 48], seed=42, with_state=False),         # 2048 tokens: the maximum
    ]
    for inp in cases:
        args = util.prefill_args(inp)
        T = args[0].shape[0]
        N = args[8].shape[0] - 1
        ref_out = torch.empty((T, 8, 128), dtype=torch.bfloat16, device="cuda")
        ref_ns = torch.empty((N, 8, 128, 128), dtype=torch.float32, device="cuda")
        _call_regular(args, ref_out, ref_ns)
        out = torch.full_like(ref_out, float("nan"))
        ns = torch.full_like(ref_ns, float("nan"))
        rc = _call_noalloc(fn, args, out, ns)
        assert rc == 0, _lib.load().gdn_status_string(rc)
        torch.cuda.synchronize()
        # the same kernels on the same inputs: the results must be bit-identical
        assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
        assert torch.equal(ns.view(torch.int32), ref_ns.view(torch.int32))


def test_noalloc_prefill_rejects_too_many_tokens():
    fn = _noalloc_fn()
    inp = gi.prefill_inputs([MAX_TOKENS + 1], seed=43, with_state=False)
    args = util.prefill_args(inp)
    out = torch.zeros((MAX_TOKENS + 1, 8, 128), dtype=torch.bfloat16, device="cuda")
    ns = torch.zeros((1, 8, 128, 128), dtype=torch.float32, device="cuda")
    rc = _call_noalloc(fn, args, out, ns)
    torch.cuda.synchronize()
    assert rc == 4  # GDN_ERR_SIZE
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(ns) == 0


def test_noalloc_prefill_rejects_too_many_sequences():
    fn = _noalloc_fn()
    inp = gi.prefill_inputs([8] * (MAX_SEQS + 1), seed=44, with_state=True)
    args = util.prefill_args(inp)
    T = args[0].shape[0]
    out = torch.zeros((T, 8, 128), dtype=torch.bfloat16, device="cuda")
    ns = torch.zeros((MAX_SEQS + 1, 8, 128, 128), dtype=torch.float32, device="cuda")
    rc = _call_noalloc(fn, args, out, ns)
    torch.cuda.synchronize()
    assert rc == 4  # GDN_ERR_SIZE
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(ns) == 0
