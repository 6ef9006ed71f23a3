"""ctypes binding of libgdn_b200.so (the C ABI in include/gdn_b200.h).

There is no fallback: if the library is missing or fails to load, every entry
point raises.  The library is loaded once per process.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

GDN_OK = 0
GDN_FLAG_QK_L2NORM = 0x4  # include/gdn_b200.h
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_U = ctypes.c_uint
_SZ = ctypes.c_size_t


class GDNError(RuntimeError):
    """A non-zero status returned by the CUDA library."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def lib_path() -> str:
    return _build.LIB_PATH


def load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = _build.LIB_PATH
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libgdn_b200.so is not built ({path}); run `python -m gdn.build` or __graft_entry__.build()")
            lib = ctypes.CDLL(path)
            lib.gdn_decode_fwd.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _P, _I, _I, _I, _I, _I, _P, _U]
            lib.gdn_decode_fwd.restype = _I
            lib.gdn_prefill_workspace_bytes.argtypes = [_I, _I, _I, _I, _I, _I]
            lib.gdn_prefill_workspace_bytes.restype = _SZ
            lib.gdn_prefill_fwd.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P, _P, _P, _SZ,
                                            _I, _I, _I, _I, _P, _U]
            lib.gdn_prefill_fwd.restype = _I
            lib.gdn_status_string.argtypes = [_I]
            lib.gdn_status_string.restype = ctypes.c_char_p
            lib.gdn_version.restype = _I
            _lib = lib
    return _lib


def check(fn: str, status: int):
    if status != GDN_OK:
        msg = load().gdn_status_string(int(status)).decode()
        raise GDNError(fn, int(status), msg)
