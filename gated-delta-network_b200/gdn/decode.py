"""Gated DeltaNet decode step on B200 (single token per sequence).

Drop-in for reference/gdn_decode_ref.py:12 (``run``) and for the
destination-passing ``kernel`` of
solutions/gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:85.
Both call ``gdn_decode_fwd`` of libgdn_b200.so on the current CUDA stream;
nothing synchronises the host unless ``scale`` is a CUDA tensor (``.item()``,
as in the reference).
"""
from __future__ import annotations

import torch

from . import _lib
from ._common import HEAD_DIM, as_dev, check_heads, cuda_device, on_device, out_ok, ptr, resolve_scale, stream_handle


def _launch(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, flags=0):
    dev = cuda_device(q, "q")
    B, T, Hq, K = q.shape
    Hk = k.shape[2]
    HV, V = v.shape[2], v.shape[3]
    # Shape contract of the reference oracle (reference/gdn_decode_ref.py:32-36), widened to any
    # head counts with HV a multiple of H.
    check_heads(Hq, Hk, HV, K, V)
    assert T == 1
    s = resolve_scale(scale)
    q_ = as_dev(q, torch.bfloat16, dev)
    k_ = as_dev(k, torch.bfloat16, dev)
    v_ = as_dev(v, torch.bfloat16, dev)
    a_ = as_dev(a, torch.bfloat16, dev)
    b_ = as_dev(b, torch.bfloat16, dev)
    A_ = as_dev(A_log, torch.float32, dev)
    d_ = as_dev(dt_bias, torch.float32, dev)
    if tuple(a_.shape[-1:]) != (HV,) or a_.numel() != B * HV or b_.numel() != B * HV:
        raise ValueError(f"a and b must hold [B, 1, {HV}] gate inputs")
    if A_.numel() != HV or d_.numel() != HV:
        raise ValueError(f"A_log and dt_bias must hold {HV} values")
    st = None
    if state is not None:
        if tuple(state.shape) != (B, HV, V, K):
            raise ValueError(f"state must be [B, {HV}, 128, 128], got {tuple(state.shape)}")
        st = as_dev(state, torch.float32, dev)
    for name, t, shape, dt in (("output", output, (B, HV * V), torch.bfloat16),
                               ("new_state", new_state, (B, HV * V * K), torch.float32)):
        if not out_ok(t, dev, dt, shape[0] * shape[1]):
            raise ValueError(f"{name} must be a contiguous {dt} CUDA tensor with {shape[0] * shape[1]} elements")
    lib = _lib.load()
    with on_device(dev):
        rc = lib.gdn_decode_fwd(ptr(q_), ptr(k_), ptr(v_), ptr(st), ptr(A_), ptr(a_), ptr(d_), ptr(b_), s,
                                ptr(output), ptr(new_state), B, Hq, HV, K, V, stream_handle(dev), flags)
    _lib.check("gdn_decode_fwd", rc)


def run(q, k, v, state, A_log, a, dt_bias, b, scale, *, use_qk_l2norm_in_kernel=False):
    """One decode step.  Returns ``(output [B,1,8,128] bf16, new_state [B,8,128,128] fp32)``.

    q, k [B,1,4,128] bf16; v [B,1,8,128] bf16; state [B,8,128,128] fp32 (k-last) or None (zeros);
    A_log, dt_bias [8] fp32; a, b [B,1,8] bf16; scale float, 0-d tensor, or None/0 (1/sqrt(128)).
    Head counts: the reference's 4 q/k heads and 8 v-heads, or any H, HV with HV a multiple of H
    (v-head hv reads q/k head hv // (HV // H)); the shapes above then read H for 4 and HV for 8.
    ``use_qk_l2norm_in_kernel=True`` (keyword only; not in the reference signature) normalises q and
    k per token and head in-kernel, x * (sum x^2 + 1e-6)^-1/2, as the reference's decode sweep
    kernel does (tests/bench_decode_sweep.py:43-46); by default q, k are used as given.
    """
    B = q.shape[0]
    dev = cuda_device(q, "q")
    HV = v.shape[2]
    output = torch.empty((B, 1, HV, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    new_state = torch.empty((B, HV, HEAD_DIM, HEAD_DIM), dtype=torch.float32, device=dev)
    _launch(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state,
            flags=_lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm_in_kernel else 0)
    return output, new_state


def kernel(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, *, use_qk_l2norm_in_kernel=False):
    """Destination-passing decode: writes ``output`` and ``new_state`` (which may be ``state`` itself)."""
    _launch(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state,
            flags=_lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm_in_kernel else 0)
