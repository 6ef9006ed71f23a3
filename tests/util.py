"""Helpers shared by the GPU parity tests: numpy inputs -> CUDA tensors, tolerance checks."""
from __future__ import annotations

import numpy as np
import torch

# Parity bar of this path: output within atol = rtol = 1e-2 (bf16 I/O, elementwise
# assert_close semantics) and final fp32 state within relative L2 error 1e-3 of the oracle.
OUT_ATOL = 1e-2
OUT_RTOL = 1e-2
STATE_REL_L2 = 1e-3


def bf16(x: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16).to(device)


def f32(x, device="cuda"):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(device)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def decode_args(inp, device="cuda"):
    return (bf16(inp["q"], device), bf16(inp["k"], device), bf16(inp["v"], device), f32(inp["state"], device),
            f32(inp["A_log"], device), bf16(inp["a"], device), f32(inp["dt_bias"], device), bf16(inp["b"], device),
            inp["scale"])


def prefill_args(inp, device="cuda", cu_dtype=torch.int32):
    return (bf16(inp["q"], device), bf16(inp["k"], device), bf16(inp["v"], device), f32(inp["state"], device),
            f32(inp["A_log"], device), bf16(inp["a"], device), f32(inp["dt_bias"], device), bf16(inp["b"], device),
            torch.from_numpy(np.asarray(inp["cu_seqlens"])).to(device=device, dtype=cu_dtype), inp["scale"])


def bf16_bits_to_f32(x):
    return (np.asarray(x, np.uint16).astype(np.uint32) << 16).view(np.float32)


def check_out(got_bits, ref_bits, atol=OUT_ATOL, rtol=OUT_RTOL):
    got = bf16_bits_to_f32(got_bits).astype(np.float64).reshape(-1)
    ref = bf16_bits_to_f32(ref_bits).astype(np.float64).reshape(-1)
    assert got.shape == ref.shape
    assert np.isfinite(got).all(), "non-finite output"
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), f"{int(bad.sum())} output elements out of tolerance; max abs err {err.max():.3e}"
    return float(err.max()) if err.size else 0.0


def check_state(got, ref, rel_l2=STATE_REL_L2):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    assert np.isfinite(got).all(), "non-finite state"
    num = np.linalg.norm(got - ref)
    den = np.linalg.norm(ref)
    rel = num / den if den > 0 else num
    assert rel <= rel_l2, f"state rel-L2 {rel:.3e} > {rel_l2:.1e}"
    return float(rel)
