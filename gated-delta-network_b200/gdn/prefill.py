"""Gated DeltaNet varlen chunked prefill on B200.

Drop-in for reference/gdn_prefill_ref.py:12 (``run``) and for the
destination-passing ``kernel`` of
solutions/gdn_prefill_qk4_v8_d128_k_last/solution/triton/fla_kernels.py:1049.
``cu_seqlens`` (int32 or int64) is read on the device only; unlike the
reference (fla_kernels.py:963, ``cu_seqlens.tolist()``) no call copies it to
the host, so a call can be captured into a CUDA graph.  The intermediate
workspace (w, u, Aqk, G: about 7.2 KB per token) comes from the torch caching
allocator, or from the caller through ``workspace=``.
"""
from __future__ import annotations

import torch

from . import _lib
from ._common import (HEAD_DIM, NUM_QK_HEADS, NUM_V_HEADS, as_dev, check_heads, cuda_device, on_device, out_ok, ptr,
                      resolve_scale, stream_handle)


def workspace_bytes(num_seqs: int, total_tokens: int, num_qk_heads: int = NUM_QK_HEADS,
                    num_v_heads: int = NUM_V_HEADS) -> int:
    return int(_lib.load().gdn_prefill_workspace_bytes(int(num_seqs), int(total_tokens), int(num_qk_heads),
                                                       int(num_v_heads), HEAD_DIM, HEAD_DIM))


def _launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, workspace=None, flags=0):
    dev = cuda_device(q, "q")
    T, Hq, K = q.shape
    Hk = k.shape[1]
    HV, V = v.shape[1], v.shape[2]
    N = cu_seqlens.shape[0] - 1
    # Shape contract of the reference oracle (reference/gdn_prefill_ref.py:33-36), widened to any
    # head counts with HV a multiple of H.
    check_heads(Hq, Hk, HV, K, V, prefill=True)
    if N < 0:
        raise ValueError("cu_seqlens must hold at least one element")
    s = resolve_scale(scale)
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError("cu_seqlens must be int32 or int64")
    cu = cu_seqlens if (cu_seqlens.is_cuda and cu_seqlens.get_device() == dev.index) else cu_seqlens.to(dev)
    if not cu.is_contiguous():
        cu = cu.contiguous()
    q_ = as_dev(q, torch.bfloat16, dev)
    k_ = as_dev(k, torch.bfloat16, dev)
    v_ = as_dev(v, torch.bfloat16, dev)
    a_ = as_dev(a, torch.bfloat16, dev)
    b_ = as_dev(b, torch.bfloat16, dev)
    A_ = as_dev(A_log, torch.float32, dev)
    d_ = as_dev(dt_bias, torch.float32, dev)
    if a_.numel() != T * HV or b_.numel() != T * HV:
        raise ValueError(f"a and b must hold [T, {HV}] gate inputs")
    if A_.numel() != HV or d_.numel() != HV:
        raise ValueError(f"A_log and dt_bias must hold {HV} values")
    st = None
    if state is not None:
        if tuple(state.shape) != (N, HV, V, K):
            raise ValueError(f"state must be [N, {HV}, 128, 128], got {tuple(state.shape)}")
        st = as_dev(state, torch.float32, dev)
    for name, t, n, dt in (("output", output, T * HV * V, torch.bfloat16),
                           ("new_state", new_state, N * HV * V * K, torch.float32)):
        if not out_ok(t, dev, dt, n):
            raise ValueError(f"{name} must be a contiguous {dt} CUDA tensor with {n} elements")
    lib = _lib.load()
    need = workspace_bytes(N, T, Hq, HV)
    if workspace is None:
        ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    else:
        ws = workspace
        if not ws.is_cuda or ws.get_device() != dev.index or ws.numel() * ws.element_size() < need:
            raise ValueError(f"workspace must be a CUDA buffer of at least {need} bytes")
    with on_device(dev):
        rc = lib.gdn_prefill_fwd(ptr(q_), ptr(k_), ptr(v_), ptr(st), ptr(A_), ptr(a_), ptr(d_), ptr(b_), ptr(cu),
                                 1 if cu.dtype == torch.int64 else 0, N, T, s, ptr(output), ptr(new_state),
                                 ptr(ws), need, Hq, HV, K, V, stream_handle(dev), flags)
    _lib.check("gdn_prefill_fwd", rc)


def read_status(workspace: torch.Tensor) -> int:
    """Device status word of the last call that used `workspace` (0 = ok; 1..3 = a bounded
    device-side wait gave up, see GDN_DEVSTATUS_* in include/gdn_b200.h).  Reads device memory,
    so it synchronises with the current stream: a debugging aid, not part of the hot path."""
    return int(workspace[:4].view(torch.int32).item())


def run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, *, use_qk_l2norm_in_kernel=False):
    """Varlen prefill.  Returns ``(output [T,8,128] bf16, new_state [N,8,128,128] fp32)``.

    q, k [T,4,128] bf16; v [T,8,128] bf16; state [N,8,128,128] fp32 or None; a, b [T,8] bf16;
    cu_seqlens [N+1] int32/int64; scale float, 0-d tensor, or None/0 (1/sqrt(128)).
    Head counts: the reference's 4 q/k heads and 8 v-heads, or any H, HV with HV a multiple of H
    (v-head hv reads q/k head hv // (HV // H)); the shapes above then read H for 4 and HV for 8.
    Tokens outside every sequence keep a zero output, and a zero-length sequence
    gets an all-zero final state, as in the reference oracle.
    ``use_qk_l2norm_in_kernel=True`` (keyword only; not in the reference signature) normalises q and
    k per token and head in-kernel, x * (sum x^2 + 1e-6)^-1/2, as the reference's decode sweep
    kernel does (tests/bench_decode_sweep.py:43-46); by default q, k are used as given.
    """
    dev = cuda_device(q, "q")
    T = q.shape[0]
    N = cu_seqlens.shape[0] - 1
    HV = v.shape[1]
    output = torch.empty((T, HV, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    new_state = torch.empty((max(N, 0), HV, HEAD_DIM, HEAD_DIM), dtype=torch.float32, device=dev)
    _launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
            flags=_lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm_in_kernel else 0)
    return output, new_state


def kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, *,
           use_qk_l2norm_in_kernel=False):
    """Destination-passing prefill: writes ``output`` and ``new_state`` (which may be ``state``)."""
    _launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
            flags=_lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm_in_kernel else 0)
