"""Host-side argument checks of the Python mirror (no GPU needed): shape violations raise
ValueError, also under ``python -O`` (they are explicit checks, not asserts)."""
import pytest

from gdn._common import check_heads


def test_check_heads_accepts_reference_family_and_supersets():
    check_heads(4, 4, 8, 128, 128, prefill=True)
    check_heads(16, 16, 32, 128, 128, prefill=True)
    check_heads(4, 4, 12, 128, 128)  # HV only needs to be a multiple of H
    check_heads(4, 4, 12, 128, 128, prefill=True)
    check_heads(1, 1, 2, 128, 128, prefill=True)  # one q/k head group of the reference family (head split)


@pytest.mark.parametrize("args", [
    (4, 2, 8, 128, 128, False),    # k with fewer heads than q: the ABI takes one H, so this must be refused
    (4, 4, 8, 64, 128, False),     # head size
    (4, 4, 8, 128, 96, False),
    (4, 4, 6, 128, 128, False),    # HV not a multiple of H
    (8, 8, 4, 128, 128, False),    # fewer v-heads than q/k heads
    (4, 4, 6, 128, 128, True),     # prefill: HV not a multiple of H
])
def test_check_heads_rejects_with_value_error(args):
    Hq, Hk, HV, K, V, prefill = args
    with pytest.raises(ValueError):
        check_heads(Hq, Hk, HV, K, V, prefill=prefill)
