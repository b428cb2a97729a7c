"""PrefixLM varlen flash attention (fwd + bwd) vs the fp32 masked-attention oracle."""
import pytest
import torch

from gpu_utils import assert_close, random_packing

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("T,H,seed,max_doc", [(2048, 2, 1, 700), (640, 1, 4, 130), (3000, 3, 5, 1500)])
def test_attention_fwd_bwd(cuda_device, causal, T, H, seed, max_doc):
    """tcgen05 forward and backward against the fp32 oracle on ragged packings: documents of
    length 1, 2, 64, 129 and 130, prefix 0 and prefix == length, T not a multiple of 128 and a
    padded tail."""
    from hrm_text_b200.models.layers import prefixlm_attention_reference
    from hrm_text_b200.ops.attention import flash_attn_varlen_prefixlm
    torch.manual_seed(seed)
    D = 128
    cu, pl, pos, total = random_packing(T, seed=seed, max_doc=max_doc)
    q, k, v = (torch.randn(T, H, D, device=cuda_device).bfloat16().requires_grad_(True) for _ in range(3))
    out = flash_attn_varlen_prefixlm(q, k, v, causal, pl.to(cuda_device), None, cu.to(cuda_device))
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = prefixlm_attention_reference(qr, kr, vr, causal, pl, cu)
    assert_close(out, ref, 2e-2, "attention fwd")
    assert out[total:].abs().max().item() == 0.0
    dout = torch.randn(T, H, D, device=cuda_device).bfloat16()
    out.backward(dout)
    ref.backward(dout.float())
    for a, b, name in ((q.grad, qr.grad, "dq"), (k.grad, kr.grad, "dk"), (v.grad, vr.grad, "dv")):
        # bf16 P and dS (relative rounding 2^-8 each) summed over up to ~1500 keys: isolated
        # elements land a few percent of the gradient's RMS away from the fp32 oracle
        assert_close(a, b, 3e-2, name, atol=0.08 * b.float().pow(2).mean().sqrt().item())
        assert a[total:].abs().max().item() == 0.0


@pytest.mark.parametrize("causal", [False, True])
def test_tcgen05_forward_matches_mma_forward(cuda_device, causal):
    """The tcgen05 forward against the mma.sync forward on a long packed batch (docs up to 4096)."""
    from hrm_text_b200.ops.attention import PackedSeq, attention_fwd
    torch.manual_seed(1)
    T, H = 8192, 3
    cu, pl, pos, total = random_packing(T, seed=7, max_doc=4096)
    packed = PackedSeq(pos.to(cuda_device), cu.to(cuda_device), pl.to(cuda_device))
    qkv = torch.randn(T, 4 * H * 128, device=cuda_device).bfloat16()
    a = attention_fwd(qkv, H, packed.schedule(causal), kernel="tcgen05")
    b = attention_fwd(qkv, H, packed.schedule(causal), kernel="mma")
    for x, y, name in zip(a, b, ("O", "Y", "lse")):
        assert_close(x[:total] if name != "lse" else x[:, :total], y[:total] if name != "lse" else y[:, :total],
                     2e-2, name)
    assert a[0][total:].abs().max().item() == 0.0


def test_tcgen05_forward_bench_shape_with_rescales(cuda_device):
    """Bench-sized launch (T=21504, 10 heads, many tiles per CTA) with key magnitudes growing
    along each document, so row maxima rise block after block and rows rescale at different
    blocks (exercises the warp-uniform lazy-rescale path)."""
    from hrm_text_b200.data.synthetic import packed_batches
    from hrm_text_b200.ops.attention import PackedSeq, attention_fwd
    torch.manual_seed(2)
    T, H = 21504, 10
    b, s = next(iter(packed_batches(T, 32768, 4096, num_batches=1, seed=5)))
    total = s["total_seqlen"]
    packed = PackedSeq(b["position_ids"].to(cuda_device), b["cu_seqlens"].to(cuda_device),
                       b["prefix_lens"].to(cuda_device))
    qkv = torch.randn(T, 4, H, 128, device=cuda_device)
    growth = 1.0 + b["position_ids"].to(cuda_device).float()[:, None, None] / 300.0
    qkv[:, 2] *= growth  # keys
    qkv = qkv.reshape(T, 4 * H * 128).bfloat16()
    a = attention_fwd(qkv, H, packed.schedule(False), kernel="tcgen05")
    ref = attention_fwd(qkv, H, packed.schedule(False), kernel="mma")
    torch.cuda.synchronize()
    from hrm_text_b200.utils.errors import check_device_errors
    check_device_errors()
    assert_close(a[0][:total], ref[0][:total], 2e-2, "O")
    assert_close(a[2][:, :total], ref[2][:, :total], 1e-3, "lse")


@pytest.mark.parametrize("causal", [False, True])
def test_tcgen05_backward_matches_mma_backward(cuda_device, causal):
    """tcgen05 backward vs mma.sync backward at the bench shape, with real RoPE tables."""
    from hrm_text_b200.data.synthetic import packed_batches
    from hrm_text_b200.models.layers import rope_tables
    from hrm_text_b200.ops.attention import PackedSeq, attention_bwd, attention_fwd
    from hrm_text_b200.utils.errors import check_device_errors
    torch.manual_seed(3)
    T, H = 21504, 10
    b, s = next(iter(packed_batches(T, 32768, 4096, num_batches=1, seed=9)))
    total = s["total_seqlen"]
    packed = PackedSeq(b["position_ids"].to(cuda_device), b["cu_seqlens"].to(cuda_device),
                       b["prefix_lens"].to(cuda_device))
    sched = packed.schedule(causal)
    qkv = torch.randn(T, 4 * H * 128, device=cuda_device).bfloat16()
    o, y, lse = attention_fwd(qkv, H, sched, kernel="mma")
    dy = torch.randn(T, H * 128, device=cuda_device).bfloat16()
    cos, sin = rope_tables(128, 4096, 10000.0, device=cuda_device)
    cos, sin = cos[:, :64].contiguous(), sin[:, :64].contiguous()
    g_tc = attention_bwd(qkv, H, sched, o, lse, dy, packed.position_ids, cos, sin, kernel="tcgen05")
    g_mma = attention_bwd(qkv, H, sched, o, lse, dy, packed.position_ids, cos, sin, kernel="mma")
    torch.cuda.synchronize()
    check_device_errors()
    for part, name in enumerate(("dgate", "dq", "dk", "dv")):
        sl = slice(part * H * 128, (part + 1) * H * 128)
        assert_close(g_tc[:total, sl], g_mma[:total, sl], 3e-2, name)
    assert g_tc[total:].abs().max().item() == 0.0
