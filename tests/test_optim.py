import math

import torch

from hrm_text_b200.optim.adam_atan2 import AdamATan2


def _manual(p, g_seq, lr, b1, b2, wd, ema):
    """Independent restatement of the update rule, step by step, in float64."""
    p = p.double().clone()
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    e = p.clone()
    for t, g in enumerate(g_seq, start=1):
        g = g.double()
        p = p * (1 - lr * wd)
        m = b1 * m + (1 - b1) * g
        v = b2 * v + (1 - b2) * g * g
        mhat_scale = lr / (1 - b1 ** t)
        denom = v.sqrt() / math.sqrt(1 - b2 ** t)
        p = p - mhat_scale * torch.atan2(m, denom)
        e = ema * e + (1 - ema) * p
    return p, e


def test_adam_atan2_matches_manual():
    torch.manual_seed(0)
    p0 = torch.randn(50)
    grads = [torch.randn(50) * 0.1 for _ in range(6)]
    param = torch.nn.Parameter(p0.clone())
    opt = AdamATan2([param], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.99)
    for g in grads:
        param.grad = g.clone()
        opt.step()
    want_p, want_e = _manual(p0, grads, 1e-2, 0.9, 0.95, 0.1, 0.99)
    torch.testing.assert_close(param.data.double(), want_p, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(opt.state[param]["param_ema"].double(), want_e, atol=1e-5, rtol=1e-5)
    assert set(opt.state[param]) == {"step", "exp_avg", "exp_avg_sq", "param_ema"}
    assert opt.state[param]["step"].item() == 6.0


def test_no_momentum_and_swap_ema():
    param = torch.nn.Parameter(torch.ones(4))
    opt = AdamATan2([param], lr=0.1, betas=(0.0, 0.9), weight_decay=0.0, ema=0.5)
    assert "exp_avg" not in opt.state[param]
    param.grad = torch.ones(4)
    opt.step()
    # atan2(g, |g|) = pi/4 after bias correction
    torch.testing.assert_close(param.data, torch.full((4,), 1 - 0.1 * math.pi / 4))
    before = param.data.clone()
    ema = opt.state[param]["param_ema"].clone()
    opt.swap_ema()
    torch.testing.assert_close(param.data, ema)
    opt.swap_ema()
    torch.testing.assert_close(param.data, before)
