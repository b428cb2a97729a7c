"""Split-K choice of the fp32 weight-gradient GEMMs (host arithmetic of the CUDA extension; no
GPU needed): the L2-sized split is only raised, and only where its units quantise badly on the
74 CTA pairs of a B200 (148 SMs)."""
import pytest
import torch  # noqa: F401  (loads libtorch for the extension)

from hrm_text_b200._native import cuda_available, cuda

PAIRS = 74

pytestmark = pytest.mark.skipif(not cuda_available(), reason="native extension not built")


def _split(s0, tiles, nk=336):
    return cuda().gemm_balanced_split(s0, tiles, PAIRS, nk)


def test_badly_quantised_gradient_gets_more_splits():
    # L o_proj gradient: 25 pair tiles; 3 splits = 75 units = two waves for one wave's work
    assert _split(3, 25) == 5


@pytest.mark.parametrize("s0,tiles", [(5, 70), (8, 140), (6, 144), (3, 70), (6, 140)])
def test_well_quantised_gradients_keep_their_split(s0, tiles):
    assert _split(s0, tiles) == s0


def test_split_never_drops_below_the_l2_split_and_respects_k():
    for s0 in range(2, 12):
        for tiles in (1, 5, 25, 70, 100, 140, 300):
            s = _split(s0, tiles)
            assert s0 <= s <= 2 * s0 + 2
    assert _split(8, 25, nk=9) <= 9
    assert _split(1, 25) == 1 and _split(0, 25) == 0
