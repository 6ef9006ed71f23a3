"""Generate the golden fixtures of the Gated DeltaNet path from the reference itself.

Run in a container that has the reference sources (it imports the reference's
own PyTorch oracles, reference/gdn_decode_ref.py::run and
reference/gdn_prefill_ref.py::run, from REF_DIR) -- not needed on a GPU box:

    python tests/golden/make_golden.py REF_DIR [CASE ...]   (no CASE: every fixture)

Inputs are regenerated from seeds by tests/golden/inputs.py; each fixture
stores a digest of its inputs (so a generator drift is detected), the full
norm of each output, its value at 4096 seeded positions and its dot products
with 8 seeded +-1 vectors.  That keeps the files small while pinning every
element of the outputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as gi  # noqa: E402

DECODE_CASES = [
    ("decode_b1", dict(B=1, seed=0, with_state=True)),
    ("decode_b4", dict(B=4, seed=1, with_state=True)),
    ("decode_b3_nostate", dict(B=3, seed=2, with_state=False)),
]

PREFILL_CASES = [
    ("prefill_32", dict(lens=[32], seed=10, with_state=False)),
    ("prefill_64", dict(lens=[64], seed=11, with_state=False)),
    ("prefill_128", dict(lens=[128], seed=12, with_state=False)),
    ("prefill_31", dict(lens=[31], seed=13, with_state=False)),
    ("prefill_65", dict(lens=[65], seed=14, with_state=False)),
    ("prefill_127", dict(lens=[127], seed=15, with_state=False)),
    ("prefill_64_64", dict(lens=[64, 64], seed=16, with_state=False)),
    ("prefill_32_96", dict(lens=[32, 96], seed=17, with_state=False)),
    ("prefill_64_128_state", dict(lens=[64, 128], seed=18, with_state=True)),
    ("prefill_128_state", dict(lens=[128], seed=19, with_state=True)),
    ("prefill_zero_len", dict(lens=[40, 0, 70], seed=20, with_state=True)),
    ("prefill_1", dict(lens=[1], seed=21, with_state=True)),
    ("prefill_200_state", dict(lens=[200], seed=22, with_state=True)),
    # long sequences: pin the oracle's fp32 accumulation where the recurrence runs longest
    ("prefill_2048_state", dict(lens=[2048], seed=23, with_state=True)),
    ("prefill_1024x2_state", dict(lens=[1024, 1024], seed=24, with_state=True)),
]


def _bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)


def _summ(name, arr):
    flat = np.asarray(arr).reshape(-1)
    idx = gi.sample_index(flat.shape[0])
    return {f"{name}_idx": idx.astype(np.int64), f"{name}_val": flat[idx],
            f"{name}_proj": gi.projections(flat.astype(np.float64) if flat.dtype != np.uint16 else gi.bf16_bits_to_f32(flat)),
            f"{name}_norm": np.array([np.linalg.norm(flat.astype(np.float64) if flat.dtype != np.uint16 else gi.bf16_bits_to_f32(flat).astype(np.float64))]),
            f"{name}_shape": np.array(np.asarray(arr).shape, np.int64)}


def main(ref_dir, only=None):
    sys.path.insert(0, os.path.join(ref_dir, "reference"))
    from gdn_decode_ref import run as ref_decode  # the reference's own oracle
    from gdn_prefill_ref import run as ref_prefill
    torch.set_num_threads(os.cpu_count() or 1)
    for name, cfg in DECODE_CASES:
        if only and name not in only:
            continue
        inp = gi.decode_inputs(**cfg)
        st = None if inp["state"] is None else torch.from_numpy(inp["state"])
        out, ns = ref_decode(_bf16(inp["q"]), _bf16(inp["k"]), _bf16(inp["v"]), st, torch.from_numpy(inp["A_log"]),
                             _bf16(inp["a"]), torch.from_numpy(inp["dt_bias"]), _bf16(inp["b"]), inp["scale"])
        rec = {"kind": np.array("decode"), "digest": np.array(gi.digest(inp)), "cfg": np.array(repr(cfg))}
        rec.update(_summ("out", out.contiguous().view(torch.int16).numpy().view(np.uint16)))
        rec.update(_summ("state", ns.numpy()))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
        print("wrote", name)
    for name, cfg in PREFILL_CASES:
        if only and name not in only:
            continue
        inp = gi.prefill_inputs(**cfg)
        st = None if inp["state"] is None else torch.from_numpy(inp["state"])
        out, ns = ref_prefill(_bf16(inp["q"]), _bf16(inp["k"]), _bf16(inp["v"]), st, torch.from_numpy(inp["A_log"]),
                              _bf16(inp["a"]), torch.from_numpy(inp["dt_bias"]), _bf16(inp["b"]),
                              torch.from_numpy(inp["cu_seqlens"]), inp["scale"])
        rec = {"kind": np.array("prefill"), "digest": np.array(gi.digest(inp)), "cfg": np.array(repr(cfg))}
        rec.update(_summ("out", out.contiguous().view(torch.int16).numpy().view(np.uint16)))
        rec.update(_summ("state", ns.numpy()))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
        print("wrote", name)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py REF_DIR [CASE ...]  (the reference checkout holding reference/gdn_*_ref.py)")
    main(sys.argv[1], set(sys.argv[2:]) or None)
