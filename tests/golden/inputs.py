"""Seeded synthetic inputs for the Gated DeltaNet path, as numpy arrays.

Distributions follow the benchmark configurations of this path: q,k ~ N(0,1)
L2-normalised over the head dimension, v ~ N(0,1), a,b ~ N(0,1) (all bf16);
A_log ~ U(0, ln 16), dt_bias ~ N(0, 0.1) (fp32 [8]); initial state ~ N(0, 0.02)
fp32 in the k-last [N, HV, V, K] layout.  bf16 tensors are returned as uint16
bit patterns (round-to-nearest-even), so the same bytes feed the CPU oracle,
the reference PyTorch code and the CUDA library.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np

H, HV, D = 4, 8, 128


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    return (np.asarray(x, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _normal(rng, shape, std=1.0):
    return (rng.standard_normal(shape) * std).astype(np.float32)


def _l2n(x):
    return x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True)).astype(np.float32)


def gates_params(rng, hv: int = HV):
    A_log = (rng.random(hv) * math.log(16.0)).astype(np.float32)
    dt_bias = _normal(rng, (hv,), 0.1)
    return A_log, dt_bias


def decode_inputs(B: int, seed: int = 0, with_state: bool = True, normalized: bool = True, h: int = H, hv: int = HV):
    """normalized=False leaves q, k as raw N(0,1) (inputs of the in-kernel L2-norm variant);
    h, hv select another head-count family (the reference's is 4 / 8)."""
    rng = np.random.default_rng(seed)
    nq = _l2n if normalized else (lambda x: x)
    q = to_bf16_bits(nq(_normal(rng, (B, 1, h, D))))
    k = to_bf16_bits(nq(_normal(rng, (B, 1, h, D))))
    v = to_bf16_bits(_normal(rng, (B, 1, hv, D)))
    a = to_bf16_bits(_normal(rng, (B, 1, hv)))
    b = to_bf16_bits(_normal(rng, (B, 1, hv)))
    A_log, dt_bias = gates_params(rng, hv)
    state = _normal(rng, (B, hv, D, D), 0.02) if with_state else None
    return dict(q=q, k=k, v=v, state=state, A_log=A_log, a=a, dt_bias=dt_bias, b=b, scale=1.0 / math.sqrt(D))


def prefill_inputs(lens, seed: int = 0, with_state: bool = True, normalized: bool = True, h: int = H, hv: int = HV):
    """normalized=False leaves q, k as raw N(0,1) (inputs of the in-kernel L2-norm variant);
    h, hv select another head-count family (the reference's is 4 / 8)."""
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in lens]
    T = int(sum(lens))
    N = len(lens)
    nq = _l2n if normalized else (lambda x: x)
    q = to_bf16_bits(nq(_normal(rng, (T, h, D))))
    k = to_bf16_bits(nq(_normal(rng, (T, h, D))))
    v = to_bf16_bits(_normal(rng, (T, hv, D)))
    a = to_bf16_bits(_normal(rng, (T, hv)))
    b = to_bf16_bits(_normal(rng, (T, hv)))
    A_log, dt_bias = gates_params(rng, hv)
    state = _normal(rng, (N, hv, D, D), 0.02) if with_state else None
    cu = np.zeros(N + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    return dict(q=q, k=k, v=v, state=state, A_log=A_log, a=a, dt_bias=dt_bias, b=b, cu_seqlens=cu,
                scale=1.0 / math.sqrt(D))


def varlen_lengths(n: int = 16, lo: int = 6, hi: int = 8192, total: int = 32768, seed: int = 0):
    """Log-uniform lengths in [lo, hi], total clipped to `total` (the varlen benchmark configuration)."""
    rng = np.random.default_rng(seed)
    lens = np.exp(rng.uniform(math.log(lo), math.log(hi), n)).astype(np.int64)
    out, acc = [], 0
    for x in lens.tolist():
        x = int(min(x, total - acc))
        out.append(max(x, 0))
        acc += out[-1]
    return out


def digest(inp: dict) -> str:
    h = hashlib.sha256()
    for key in sorted(inp):
        val = inp[key]
        if val is None:
            h.update(key.encode() + b":none")
        elif isinstance(val, np.ndarray):
            h.update(key.encode() + str(val.dtype).encode() + str(val.shape).encode() + val.tobytes())
        else:
            h.update(key.encode() + repr(val).encode())
    return h.hexdigest()


def sample_index(n: int, count: int = 4096, seed: int = 1234) -> np.ndarray:
    count = min(n, count)
    return np.sort(np.random.default_rng(seed).choice(n, size=count, replace=False))


def projections(x: np.ndarray, nproj: int = 8, seed: int = 4321) -> np.ndarray:
    """Dot products of the flattened array with `nproj` seeded +-1 vectors (float64)."""
    flat = np.asarray(x, np.float64).reshape(-1)
    rng = np.random.default_rng(seed)
    out = np.empty(nproj, np.float64)
    for i in range(nproj):
        s = rng.integers(0, 2, flat.shape[0]).astype(np.float64) * 2.0 - 1.0
        out[i] = float(flat @ s)
    return out
