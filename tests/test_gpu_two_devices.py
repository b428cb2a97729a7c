"""One process, two GPUs: kernel attributes (shared-memory limits, cluster occupancy) are set
per device, so the first launch on cuda:1 after work on cuda:0 must succeed and be correct.
Skipped with fewer than 2 GPUs."""
import pytest
import torch

from gpu_utils import assert_close, random_packing

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemm_and_attention_on_second_device_after_first():
    from hrm_text_b200.models.layers import prefixlm_attention_reference
    from hrm_text_b200.ops import gemm as G
    from hrm_text_b200.ops.attention import PackedSeq, attention_bwd, attention_fwd
    from hrm_text_b200.utils.errors import check_device_errors
    T, H = 1536, 2
    cu, pl, pos, total = random_packing(T, seed=11, max_doc=600)
    for index in (0, 1, 0):
        dev = torch.device("cuda", index)
        with torch.cuda.device(dev):
            torch.manual_seed(index)
            x = torch.randn(2048, 1280, device=dev).bfloat16()  # CTA-pair GEMM
            w = torch.randn(1536, 1280, device=dev).bfloat16()
            assert_close(G.linear(x, w), x.float() @ w.float().T, 1e-2, f"gemm on {dev}")
            xs, ws = x[:200], w[:256]  # single-CTA GEMM
            assert_close(G.linear(xs, ws), xs.float() @ ws.float().T, 1e-2, f"small gemm on {dev}")
            packed = PackedSeq(pos.to(dev), cu.to(dev), pl.to(dev))
            qkv = torch.randn(T, 4 * H * 128, device=dev).bfloat16()
            o, y, lse = attention_fwd(qkv, H, packed.schedule(False))
            q, k, v = (qkv[:, (i + 1) * H * 128:(i + 2) * H * 128].float().view(T, H, 128) for i in range(3))
            ref = prefixlm_attention_reference(q, k, v, False, pl, cu).reshape(T, H * 128)
            assert_close(o, ref, 2e-2, f"attention on {dev}")
            cos = torch.ones(1, 64, device=dev)
            sin = torch.zeros(1, 64, device=dev)
            dy = torch.randn(T, H * 128, device=dev).bfloat16()
            g = attention_bwd(qkv, H, packed.schedule(False), o, lse, dy, torch.zeros_like(packed.position_ids),
                              cos, sin)
            assert torch.isfinite(g.float()).all().item()
            torch.cuda.synchronize(dev)
            check_device_errors()
