"""CPU oracle for the Gated DeltaNet decode / prefill path.

TEST INFRASTRUCTURE ONLY.  The shipped library never imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and ``--impl reference`` arm) use it, as the checker and as the timed CPU
baseline.

``decode`` / ``prefill`` wrap ``gdn_oracle.c`` (a plain-C restatement of
reference/gdn_decode_ref.py:12-83 and reference/gdn_prefill_ref.py:12-91)
through ctypes.  Inputs are numpy arrays: bf16 tensors travel as ``uint16``
bit patterns, fp32 as ``float32``.  The library is built on first use with
``make`` (gcc + OpenMP) into ``oracle/_build/``.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libgdn_oracle.so")
_lock = threading.Lock()
_lib = None

H, HV, D = 4, 8, 128


def build(force: bool = False) -> str:
    """Compile gdn_oracle.c into oracle/_build/libgdn_oracle.so (idempotent)."""
    src = os.path.join(_HERE, "gdn_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "all"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            build()
            lib = ctypes.CDLL(_LIB_PATH)
            p = ctypes.c_void_p
            lib.gdn_oracle_decode.argtypes = [p, p, p, p, p, p, p, p, ctypes.c_float, p, p, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int]
            lib.gdn_oracle_decode.restype = ctypes.c_int
            lib.gdn_oracle_prefill.argtypes = [p, p, p, p, p, p, p, p, p, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                               p, p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
            lib.gdn_oracle_prefill.restype = ctypes.c_int
            lib.gdn_oracle_max_threads.restype = ctypes.c_int
            _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().gdn_oracle_max_threads())


def _c(x, dtype):
    a = np.ascontiguousarray(x, dtype=dtype)
    return a, a.ctypes.data_as(ctypes.c_void_p)


def _scale(scale):
    if scale is None or float(scale) == 0.0:
        return 1.0 / math.sqrt(D)
    return float(scale)


def decode(q, k, v, state, A_log, a, dt_bias, b, scale, threads: int = 0, qk_l2norm: bool = False):
    """Decode step.  q,k [B,1,4,128] u16; v [B,1,8,128] u16; state [B,8,128,128] f32 or None;
    a,b [B,1,8] u16.  Returns (out [B,1,8,128] u16 bf16 bits, new_state [B,8,128,128] f32).
    qk_l2norm: normalise q, k per token and head first (the in-kernel L2-norm variant)."""
    lib = _load()
    B = int(q.shape[0])
    Hq, Hv = int(q.shape[-2]), int(v.shape[-2])
    keep = []
    args = []
    for x, dt in ((q, np.uint16), (k, np.uint16), (v, np.uint16)):
        arr, ptr = _c(x, dt); keep.append(arr); args.append(ptr)
    if state is None:
        args.append(None)
    else:
        arr, ptr = _c(state, np.float32); keep.append(arr); args.append(ptr)
    for x, dt in ((A_log, np.float32), (a, np.uint16), (dt_bias, np.float32), (b, np.uint16)):
        arr, ptr = _c(x, dt); keep.append(arr); args.append(ptr)
    out = np.zeros((B, 1, Hv, D), np.uint16)
    new_state = np.zeros((B, Hv, D, D), np.float32)
    rc = lib.gdn_oracle_decode(*args, _scale(scale), out.ctypes.data_as(ctypes.c_void_p),
                               new_state.ctypes.data_as(ctypes.c_void_p), B, int(threads), int(bool(qk_l2norm)), Hq, Hv)
    if rc != 0:
        raise ValueError(f"gdn_oracle_decode failed ({rc})")
    return out, new_state


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, threads: int = 0, qk_l2norm: bool = False):
    """Varlen prefill.  q,k [T,4,128] u16; v [T,8,128] u16; state [N,8,128,128] f32 or None;
    a,b [T,8] u16; cu_seqlens [N+1] int.  Returns (out [T,8,128] u16, new_state [N,8,128,128] f32).
    qk_l2norm: normalise q, k per token and head first (the in-kernel L2-norm variant)."""
    lib = _load()
    T = int(q.shape[0])
    Hq, Hv = int(q.shape[-2]), int(v.shape[-2])
    cu = np.ascontiguousarray(np.asarray(cu_seqlens).astype(np.int64))
    N = int(cu.shape[0]) - 1
    keep = [cu]
    args = []
    for x, dt in ((q, np.uint16), (k, np.uint16), (v, np.uint16)):
        arr, ptr = _c(x, dt); keep.append(arr); args.append(ptr)
    if state is None:
        args.append(None)
    else:
        arr, ptr = _c(state, np.float32); keep.append(arr); args.append(ptr)
    for x, dt in ((A_log, np.float32), (a, np.uint16), (dt_bias, np.float32), (b, np.uint16)):
        arr, ptr = _c(x, dt); keep.append(arr); args.append(ptr)
    out = np.zeros((T, Hv, D), np.uint16)
    new_state = np.zeros((max(N, 0), Hv, D, D), np.float32)
    rc = lib.gdn_oracle_prefill(*args, cu.ctypes.data_as(ctypes.c_void_p), N, T, _scale(scale),
                                out.ctypes.data_as(ctypes.c_void_p), new_state.ctypes.data_as(ctypes.c_void_p),
                                int(threads), int(bool(qk_l2norm)), Hq, Hv)
    if rc != 0:
        raise ValueError(f"gdn_oracle_prefill failed ({rc})")
    return out, new_state


def bf16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    return (np.asarray(x, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)
