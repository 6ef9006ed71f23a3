"""The C-ABI library: it loads, exports every symbol of include/gdn_b200.h, and its
host-side validation answers without touching a GPU (CPU-only tests)."""
import ctypes
import os
import re

import pytest

from gdn import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(gdn_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_library_exports_every_header_symbol(lib):
    syms = header_symbols()
    assert {"gdn_decode_fwd", "gdn_prefill_fwd", "gdn_prefill_workspace_bytes"} <= set(syms)
    for s in syms:
        assert hasattr(lib, s), f"missing export {s}"


def test_version_and_status_strings(lib):
    assert lib.gdn_version() >= 100
    for code in range(0, 8):
        assert lib.gdn_status_string(code)
    assert b"unknown" in lib.gdn_status_string(99)


def test_workspace_bytes(lib):
    ws = lambda n, t: lib.gdn_prefill_workspace_bytes(n, t, 4, 8, 128, 128)
    assert 0 < ws(1, 0) <= 1 << 20  # chunk table and status word only
    w1 = ws(1, 1024)
    # w (bf16) + u (f32) + Aqk (bf16, 64 wide) + G (f32), per token and v-head
    assert w1 >= 1024 * 8 * (128 * 2 + 128 * 4 + 64 * 2 + 4)
    assert w1 % 256 == 0
    assert ws(16, 32768) > ws(1, 8192)
    assert lib.gdn_prefill_workspace_bytes(1, 1024, 4, 8, 64, 128) == 0  # unsupported shape
    # other head counts: HV a multiple of H; the per-head regions scale with HV (the
    # segment regions of the segmented route also with the segment length, chosen per HV)
    ws32 = lib.gdn_prefill_workspace_bytes(1, 1024, 16, 32, 128, 128)
    assert 2.5 * w1 < ws32 < 4.5 * w1
    assert lib.gdn_prefill_workspace_bytes(1, 1024, 4, 12, 128, 128) > 0
    assert lib.gdn_prefill_workspace_bytes(1, 1024, 1, 2, 128, 128) > 0
    assert lib.gdn_prefill_workspace_bytes(1, 1024, 3, 8, 128, 128) == 0
    assert lib.gdn_prefill_workspace_bytes(-1, 1024, 4, 8, 128, 128) == 0


def _decode(lib, B=1, H=4, HV=8, K=128, V=128, ptrs=None, flags=0):
    p = ptrs or [16] * 11
    return lib.gdn_decode_fwd(p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7], 1.0, p[9], p[10], B, H, HV, K, V,
                              None, flags)


def test_decode_rejects_bad_shapes_without_gpu(lib):
    assert _decode(lib, H=3) == 2  # HV must be a multiple of H
    assert _decode(lib, H=0) == 2
    assert _decode(lib, HV=2) == 2  # fewer v-heads than q/k heads
    assert _decode(lib, H=128, HV=128) == 2  # above GDN_MAX_QK_HEADS
    assert _decode(lib, K=64) == 2
    assert _decode(lib, B=-1) == 4


def test_decode_rejects_null_and_misaligned(lib):
    p = [16] * 11
    p[0] = None
    assert _decode(lib, ptrs=p) == 1
    p = [16] * 11
    p[10] = 24  # new_state not 16-byte aligned
    assert _decode(lib, ptrs=p) == 3
    p = [16] * 11
    p[3] = None  # NULL state is allowed (zeros); B=0 launches nothing
    assert _decode(lib, B=0, ptrs=p) == 0


def _prefill(lib, N=1, T=64, ws=256, ws_bytes=1 << 30, state=None, cu64=0, H=4, HV=8):
    a = 256
    return lib.gdn_prefill_fwd(a, a, a, state, a, a, a, a, a, cu64, N, T, 1.0, a, a, ws, ws_bytes, H, HV, 128, 128,
                               None, 0)


def test_prefill_rejects_bad_arguments_without_gpu(lib):
    assert _prefill(lib, H=3) == 2  # HV must be a multiple of H
    assert _prefill(lib, HV=6) == 2  # HV must be a multiple of H
    assert _prefill(lib, N=-1) == 4
    assert _prefill(lib, T=-5) == 4
    assert _prefill(lib, N=0) == 0  # nothing to do
    assert _prefill(lib, ws=None) == 5
    assert _prefill(lib, ws=256 + 16) == 5  # workspace must be 256-byte aligned
    assert _prefill(lib, ws_bytes=1024) == 5  # too small
    assert _prefill(lib, cu64=2) == 4
    assert _prefill(lib, state=24) == 3


def test_python_entry_points_fail_loudly_on_cpu_tensors():
    import torch
    import gdn

    q = torch.zeros(1, 1, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        gdn.decode.run(q, q, torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16), None, torch.zeros(8),
                       torch.zeros(1, 1, 8, dtype=torch.bfloat16), torch.zeros(8),
                       torch.zeros(1, 1, 8, dtype=torch.bfloat16), None)
    qp = torch.zeros(4, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        gdn.prefill.run(qp, qp, torch.zeros(4, 8, 128, dtype=torch.bfloat16), None, torch.zeros(8),
                        torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(8),
                        torch.zeros(4, 8, dtype=torch.bfloat16), torch.tensor([0, 4], dtype=torch.int32), None)


def test_scale_resolution():
    import math
    import torch
    from gdn._common import resolve_scale

    assert resolve_scale(None) == pytest.approx(1 / math.sqrt(128))
    assert resolve_scale(0.0) == pytest.approx(1 / math.sqrt(128))
    assert resolve_scale(torch.tensor(0.5)) == 0.5
    assert resolve_scale(2) == 2.0


def test_prefill_gate_pointer_alignment_depends_on_head_count(lib):
    """a and b are TMA tiles (16-byte aligned) when HV is a multiple of 8, plain bf16 loads (2-byte
    aligned) otherwise; the check runs before any device work, so no GPU is needed."""
    def call(gate_ptr, H, HV):
        p = 256
        return lib.gdn_prefill_fwd(p, p, p, None, p, gate_ptr, p, gate_ptr, p, 0, 1, 64, 1.0, p, p, 256, 1 << 30,
                                   H, HV, 128, 128, None, 0)
    assert call(258, 4, 8) == 3   # 8 v-heads: gate tiles need 16-byte alignment
    assert call(258, 1, 2) != 3   # 2 v-heads: 2-byte alignment is enough
    assert call(257, 1, 2) == 3   # but not an odd address
