"""PrefixLM varlen flash attention (fwd + bwd) vs the fp32 masked-attention oracle."""
import pytest
import torch

from gpu_utils import assert_close, random_packing

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
def test_attention_fwd_bwd(cuda_device, causal):
    from hrm_text_b200.models.layers import prefixlm_attention_reference
    from hrm_text_b200.ops.attention import flash_attn_varlen_prefixlm
    torch.manual_seed(0)
    T, H, D = 2048, 2, 128
    cu, pl, pos, total = random_packing(T, seed=1)
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
        assert_close(a, b, 3e-2, name)
        assert a[total:].abs().max().item() == 0.0
