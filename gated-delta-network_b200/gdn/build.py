"""Compile the sm_100a CUDA library (csrc/*.cu) into gdn/_lib/libgdn_b200.so, in-tree.

    python -m gdn.build            (from the gated-delta-network_b200 directory)

nvcc cross-compiles for sm_100a without a GPU.  The library has no torch
dependency: it exports the C ABI declared in include/gdn_b200.h.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(PKG_DIR), "csrc")
INCLUDE = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libgdn_b200.so")
SOURCES = ["api.cu", "decode.cu", "prefill_host.cu", "prefill_prep.cu", "prefill_scan.cu", "prefill_scan_tc.cu", "prefill_short.cu", "prefill_short_rec.cu", "prefill_seg.cu", "noalloc.cu"]
HEADERS = ["common.cuh", "kernels.cuh", "sm100.cuh", "prefill_kernels.cuh", "dbg.cuh"]

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libgdn_b200.so")
    return cand


def _inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(INCLUDE, "gdn_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []), "-I", INCLUDE, "-o", tmp,
           *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
