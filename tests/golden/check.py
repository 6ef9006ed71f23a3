"""Compare an implementation's outputs against a golden fixture (see make_golden.py)."""
from __future__ import annotations

import ast
import glob
import os

import numpy as np

from . import inputs as gi

HERE = os.path.dirname(os.path.abspath(__file__))


def fixtures(kind=None):
    out = []
    for path in sorted(glob.glob(os.path.join(HERE, "*.npz"))):
        fx = dict(np.load(path))
        if kind is None or str(fx["kind"]) == kind:
            out.append((os.path.splitext(os.path.basename(path))[0], fx))
    return out


def regen(fx):
    cfg = ast.literal_eval(str(fx["cfg"]))
    inp = gi.decode_inputs(**cfg) if str(fx["kind"]) == "decode" else gi.prefill_inputs(**cfg)
    assert gi.digest(inp) == str(fx["digest"]), "input generator drifted from the one that made the fixture"
    return inp


def _as_f64(name, arr):
    flat = np.asarray(arr).reshape(-1)
    if flat.dtype == np.uint16:
        return gi.bf16_bits_to_f32(flat).astype(np.float64)
    return flat.astype(np.float64)


def compare(fx, name, arr, atol, rtol, proj_rtol):
    """Check `arr` (uint16 bf16 bits or float32) against the fixture summary `name`.

    Sampled elements: |x - ref| <= atol + rtol*|ref| (assert_close semantics).
    Projections on +-1 vectors: |p - p_ref| <= proj_rtol * ||ref||_2.
    Returns a dict of the observed errors.
    """
    assert tuple(np.asarray(arr).shape) == tuple(fx[f"{name}_shape"].tolist()), (name, np.asarray(arr).shape)
    x = _as_f64(name, arr)
    idx = fx[f"{name}_idx"]
    ref_val = _as_f64(name, fx[f"{name}_val"])
    got = x[idx]
    err = np.abs(got - ref_val)
    bad = err > atol + rtol * np.abs(ref_val)
    assert not np.isnan(got).any(), f"{name}: NaN in output"
    assert not bad.any(), f"{name}: {bad.sum()} sampled elements out of tolerance, max err {err.max():.3e}"
    proj = gi.projections(x)
    norm = float(fx[f"{name}_norm"][0])
    perr = np.abs(proj - fx[f"{name}_proj"]).max()
    assert perr <= proj_rtol * max(norm, 1e-30), f"{name}: projection err {perr:.3e} vs norm {norm:.3e}"
    return {"max_sample_err": float(err.max()) if err.size else 0.0, "proj_err_rel": perr / max(norm, 1e-30)}
