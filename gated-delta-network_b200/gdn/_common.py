"""Argument normalisation shared by the decode and prefill entry points."""
from __future__ import annotations

import contextlib
import math

import torch

NUM_QK_HEADS = 4
NUM_V_HEADS = 8
HEAD_DIM = 128


def resolve_scale(scale) -> float:
    """None / 0 -> 1/sqrt(128) (reference/gdn_decode_ref.py:38-39); 0-d tensors -> .item()
    (solutions/gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:92-93)."""
    if isinstance(scale, torch.Tensor):
        scale = scale.item()
    if scale is None or float(scale) == 0.0:
        return 1.0 / math.sqrt(HEAD_DIM)
    return float(scale)


def check_heads(Hq: int, Hk: int, HV: int, K: int, V: int, prefill: bool = False) -> None:
    """The reference asserts 4 q/k heads, 8 v-heads and head size 128
    (reference/gdn_decode_ref.py:32-36, reference/gdn_prefill_ref.py:33-36).  This library
    accepts any head counts with HV a multiple of H (v-head hv reads q/k head hv // (HV // H));
    the head size stays 128."""
    if Hk != Hq:
        raise ValueError(f"q and k must have the same number of heads (got {Hq} and {Hk})")
    if K != HEAD_DIM or V != HEAD_DIM:
        raise ValueError(f"head size must be {HEAD_DIM} (got K={K}, V={V})")
    if not (1 <= Hq <= HV and HV % Hq == 0):
        raise ValueError(f"v-heads must be a multiple of the q/k heads (got H={Hq}, HV={HV})")


def cuda_device(t: torch.Tensor, name: str) -> torch.device:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); there is no CPU path")
    return t.device


def as_dev(t: torch.Tensor, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """Contiguous, 16-byte aligned tensor of `dtype` on `device` (copies only when needed: the
    library reads its inputs with TMA tile copies, which need 16-byte aligned bases)."""
    if (t.dtype is dtype and t.is_cuda and t.get_device() == device.index and t.is_contiguous()
            and not t.data_ptr() & 15):
        return t  # the common case: nothing to convert (checked with cheap attribute reads)
    if t.device != device or t.dtype != dtype:
        t = t.to(device=device, dtype=dtype)
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def ptr(t):
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """cudaStream_t of the current torch stream on `device`."""
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def on_device(device: torch.device):
    """Make `device` current for the library call (a no-op context when it already is)."""
    if torch.cuda.current_device() == device.index:
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def out_ok(t, device: torch.device, dtype: torch.dtype, numel: int) -> bool:
    return (isinstance(t, torch.Tensor) and t.is_cuda and t.get_device() == device.index and t.dtype is dtype
            and t.is_contiguous() and t.numel() == numel)
