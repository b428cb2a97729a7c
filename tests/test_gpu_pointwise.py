"""RMSNorm / embedding / cross-entropy finalisation / AdamATan2 kernels vs fp32 torch."""
import math

import pytest
import torch
import torch.nn.functional as F

from gpu_utils import assert_close

pytestmark = pytest.mark.gpu


def test_rmsnorm_fwd_bwd(cuda_device):
    from hrm_text_b200.ops.block import rmsnorm, rmsnorm_bwd
    torch.manual_seed(0)
    T, H = 300, 1280
    x = torch.randn(T, H, device=cuda_device).bfloat16()
    inj = torch.randn(T, H, device=cuda_device).bfloat16()
    y, rstd, s = rmsnorm(x, 1e-6, inj)
    s_ref = (x.float() + inj.float()).bfloat16().float()
    assert_close(s, s_ref, 1e-2, "sum")
    y_ref = F.rms_norm(s_ref, (H,), eps=1e-6)
    assert_close(y, y_ref, 1e-2, "rmsnorm fwd")
    dy = torch.randn(T, H, device=cuda_device).bfloat16()
    dres = torch.randn(T, H, device=cuda_device).bfloat16()
    dx = rmsnorm_bwd(dy, s, rstd, dres)
    sr = s_ref.clone().requires_grad_(True)
    F.rms_norm(sr, (H,), eps=1e-6).backward(dy.float())
    assert_close(dx, sr.grad + dres.float(), 2e-2, "rmsnorm bwd")


def test_embedding(cuda_device):
    from hrm_text_b200.ops.embedding import scaled_embedding
    torch.manual_seed(0)
    V, H, T = 1000, 512, 777
    w = torch.randn(V, H, device=cuda_device).bfloat16()
    w.main_grad = torch.zeros(V, H, device=cuda_device)
    ids = torch.randint(0, V, (T,), device=cuda_device, dtype=torch.int32)
    wr = w.detach().float().requires_grad_(True)
    out = scaled_embedding(ids, w.requires_grad_(True), 3.0)
    ref = 3.0 * F.embedding(ids.long(), wr)
    assert_close(out, ref, 1e-2, "embedding fwd")
    g = torch.randn(T, H, device=cuda_device).bfloat16()
    out.backward(g)
    ref.backward(g.float())
    assert_close(w.main_grad, wr.grad, 1e-3, "embedding bwd")


def test_adam_atan2_kernel(cuda_device):
    from hrm_text_b200._native import cuda
    from hrm_text_b200.optim.adam_atan2 import reference_update
    torch.manual_seed(0)
    n = 100003
    p = torch.randn(n, device=cuda_device)
    g = torch.randn(n, device=cuda_device) * 1e-3
    m = torch.randn(n, device=cuda_device) * 1e-3
    v = torch.rand(n, device=cuda_device) * 1e-6
    e = p.clone()
    out16 = torch.empty(n, dtype=torch.bfloat16, device=cuda_device)
    refs = [t.clone() for t in (p, m, v, e)]
    lr, b1, b2, wd, ema, step = 2e-4, 0.9, 0.95, 0.1, 0.999, 7.0
    hyper = torch.tensor([lr, 1 / (1 - b1 ** step), 1 / math.sqrt(1 - b2 ** step), step], device=cuda_device)
    cuda().adam_atan2(p, g, m, v, e, out16, hyper, b1, b2, wd, ema)
    reference_update(refs[0], g, refs[1], refs[2], refs[3], step, lr, b1, b2, wd, ema)
    for a, b, name in zip((p, m, v, e), refs, ("param", "exp_avg", "exp_avg_sq", "ema")):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-5, msg=name)
    torch.testing.assert_close(out16.float(), p.bfloat16().float())
