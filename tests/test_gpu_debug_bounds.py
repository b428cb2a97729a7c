"""The bounds-check build (``HRM_DEBUG_BOUNDS=1 python setup.py build_ext --inplace``).

Each case hands a kernel an index outside its tensor and checks that the debug build records
"bounds check failed" (code 4) with the expected site in the device error word and skips the
access. These cases are out-of-bounds accesses in the regular build, so the whole module is
skipped unless the loaded extension reports ``debug_bounds_build()``.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def debug_build(cuda_device):
    from hrm_text_b200._native import cuda
    if not cuda().debug_bounds_build():
        pytest.skip("the loaded extension is the regular build (HRM_DEBUG_BOUNDS not set)")
    from hrm_text_b200.utils.errors import error_word
    error_word().zero_()
    return cuda_device


def _word():
    from hrm_text_b200.utils.errors import error_word
    torch.cuda.synchronize()
    w = error_word()
    host = w.cpu().tolist()
    w.zero_()
    return host


def test_embedding_id_past_the_table(debug_build):
    from hrm_text_b200.ops.embedding import scaled_embedding
    w = torch.randn(64, 256, device=debug_build).bfloat16()
    ids = torch.tensor([1, 5, 64, 2], dtype=torch.int32, device=debug_build)
    scaled_embedding(ids, w, 1.0)
    code, site = _word()[:2]
    assert (code, site) == (4, 95)


def test_rope_position_past_the_tables(debug_build):
    from hrm_text_b200.ops import gemm as G
    x = torch.randn(256, 256, device=debug_build).bfloat16()
    w = torch.randn(1024, 256, device=debug_build).bfloat16()
    cos = torch.ones(16, 64, device=debug_build)
    sin = torch.zeros(16, 64, device=debug_build)
    pos = torch.arange(256, dtype=torch.int32, device=debug_build)  # rows 16.. are past the tables
    G.linear_rope(x, w, pos, cos, sin, 256, 768)
    code, site = _word()[:2]
    assert (code, site) == (4, 80)


def test_decode_length_past_the_cache(debug_build):
    from hrm_text_b200._native import cuda
    B, H, S = 2, 2, 64
    gqkv = torch.randn(B, 4 * H * 128, device=debug_build).bfloat16()
    kc = torch.zeros(B, S, H, 128, device=debug_build).bfloat16()
    vc = torch.zeros_like(kc)
    lengths = torch.tensor([3, S], dtype=torch.int32, device=debug_build)  # the second row is full
    cuda().decode_attention_gqkv(gqkv, H, kc, vc, lengths)
    code, site = _word()[:2]
    assert code == 4 and site in (90, 91)


def test_attention_tile_outside_the_packing(debug_build):
    from hrm_text_b200.ops.attention import attention_fwd
    T, H = 512, 1
    qkv = torch.randn(T, 4 * H * 128, device=debug_build).bfloat16()
    sched = torch.zeros(8 + 8 * 4, dtype=torch.int32, device=debug_build)
    sched[0] = 1      # one forward tile ...
    sched[2] = T      # ... of T packed tokens
    sched[8:12] = torch.tensor([400, 200, 0, 0], dtype=torch.int32)  # doc [400, 600) is past T
    attention_fwd(qkv, H, sched)
    code, site = _word()[:2]
    assert (code, site) == (4, 100)
