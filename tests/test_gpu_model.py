"""Fused transformer block / full HRM step on the GPU vs the fp32 torch oracle."""
import pytest
import torch

from gpu_utils import assert_close, random_packing

pytestmark = pytest.mark.gpu


def _tiny_cfg(**kw):
    from hrm_text_b200.runtime.factory import arch_preset
    arch = arch_preset("hrm", "L") | dict(n_layers=4, hidden_size=256, num_heads=2, H_cycles=2, L_cycles=2,
                                          bp_max_steps=3)
    return arch | dict(vocab_size=1024, max_seq_len=1024) | kw


def _batch(T, device, seed=0):
    cu, pl, pos, total = random_packing(T, seed=seed, max_doc=400)
    g = torch.Generator().manual_seed(seed)
    inputs = torch.randint(0, 1024, (T,), generator=g, dtype=torch.int32)
    labels = torch.randint(0, 1024, (T,), generator=g, dtype=torch.int32)
    labels[total:] = -100
    labels[::5] = -100
    causal = (cu[1:] - cu[:-1]).clamp(min=0)
    return {k: v.to(device) for k, v in dict(inputs=inputs, labels=labels, position_ids=pos, prefix_lens=pl,
                                               causal_lens=causal, cu_seqlens=cu).items()}


def test_block_matches_oracle(cuda_device):
    from hrm_text_b200.models.transformer import Transformer, TransformerConfig
    torch.manual_seed(0)
    cfg = TransformerConfig(max_seq_len=1024, n_layers=2, hidden_size=256, num_heads=2, expansion=4,
                            init_type="lecun_normal", norm_type="pre", norm_eps=1e-6, pos_emb_type="rope",
                            rope_theta=10000.0)
    ref = Transformer(cfg).to(cuda_device)
    fused = Transformer(cfg).to(cuda_device)
    fused.load_state_dict(ref.state_dict())
    fused = fused.to(torch.bfloat16)
    b = _batch(1024, cuda_device)
    seq = dict(position_ids=b["position_ids"], prefix_lens=b["prefix_lens"], cu_seqlens=b["cu_seqlens"])
    x = torch.randn(1024, 256, device=cuda_device)
    inj = torch.randn(1024, 256, device=cuda_device)
    xb, ib = x.bfloat16().requires_grad_(True), inj.bfloat16().requires_grad_(True)
    out = fused(xb, injection=ib, **dict(seq))
    # oracle in fp32 on bf16-rounded weights
    for p in ref.parameters():
        p.data = p.data.bfloat16().float()
    from hrm_text_b200.models.common import oracle_mode
    xr, ir = xb.detach().float().requires_grad_(True), ib.detach().float().requires_grad_(True)
    with oracle_mode():
        out_ref = ref(xr, injection=ir, **dict(seq))
    assert_close(out, out_ref, 5e-2, "block fwd")
    g = torch.randn_like(out_ref)
    out.backward(g.bfloat16())
    out_ref.backward(g)
    assert_close(xb.grad, xr.grad, 8e-2, "block dx")
    for (n, pf), pr in zip(fused.named_parameters(), ref.parameters()):
        assert_close(pf.grad, pr.grad, 8e-2, n)


def test_hrm_train_step_gpu_vs_cpu(cuda_device):
    from hrm_text_b200.runtime.engine import TrainEngine
    from hrm_text_b200.runtime.factory import build_model
    cfg = _tiny_cfg()
    torch.manual_seed(0)
    m_gpu = build_model(cfg, cuda_device)
    torch.manual_seed(0)
    m_cpu = build_model(cfg, "cpu")
    m_cpu.load_state_dict(m_gpu.state_dict())
    for p in m_cpu.parameters():
        p.data = p.data.bfloat16().float()
    for p in m_gpu.parameters():
        p.data = p.data.bfloat16().float()
    eg = TrainEngine(m_gpu, beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.999)
    ec = TrainEngine(m_cpu, beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.999)
    start = ec.params.master.clone()
    torch.testing.assert_close(eg.params.master.cpu(), start)
    for step in range(3):
        b = _batch(1024, cuda_device, seed=step)
        lg, mg = eg.train_step(b, lr=1e-3, bp_steps=3)
        lc, mc = ec.train_step({k: v.cpu() for k, v in b.items()}, lr=1e-3, bp_steps=3)
        assert abs(lg.item() - lc.item()) < 0.02 * abs(lc.item()), (step, lg.item(), lc.item())
    # Parameters: AdamATan2's early steps are nearly sign updates (|step| ~ lr), so elements whose
    # gradient is at bf16 noise level may legitimately move the other way; compare each
    # parameter's total update by direction and size instead of element by element.
    torch.cuda.synchronize()
    for s in ec.params.slots:
        dc = (ec.params.master_view(s) - start[s.shard_off: s.shard_off + s.shard_numel].view_as(
            ec.params.master_view(s))).flatten().double()
        dg = (eg.params.master_view(s).cpu() - start[s.shard_off: s.shard_off + s.shard_numel].view_as(
            ec.params.master_view(s))).flatten().double()
        if dc.norm() == 0:
            assert dg.norm() == 0, s.fqn
            continue
        cos = torch.dot(dc, dg) / (dc.norm() * dg.norm() + 1e-30)
        ratio = dg.norm() / dc.norm()
        assert cos > 0.9 and abs(ratio - 1) < 0.1, (s.fqn, float(cos), float(ratio))
    # the GPU compute weights are the bf16 rounding of its master weights
    for s in eg.params.slots:
        full = eg.params.master_view(s).reshape(-1)[: s.numel].view(s.shape)
        assert torch.equal(eg.params.full_view(eg.params.compute, s), full.bfloat16()), s.fqn


def test_graphed_step_matches_eager(cuda_device):
    from hrm_text_b200.runtime.engine import GraphedTrainStep, TrainEngine
    from hrm_text_b200.runtime.factory import build_model
    cfg = _tiny_cfg()
    losses = []
    for graphed in (False, True):
        torch.manual_seed(0)
        m = build_model(cfg, cuda_device)
        eng = TrainEngine(m, beta1=0.9, beta2=0.95, weight_decay=0.1, ema=None)
        runner = GraphedTrainStep(eng, _batch(1024, "cpu")) if graphed else None
        out = []
        for step in range(4):
            b = _batch(1024, "cpu", seed=step)
            if graphed:
                loss, _ = runner(b, lr=1e-3, bp_steps=3)
            else:
                loss, _ = eng.train_step({k: v.to(cuda_device) for k, v in b.items()}, lr=1e-3, bp_steps=3)
            out.append(loss.item())
        losses.append(out)
    for a, b in zip(*losses):
        assert abs(a - b) < 1e-2 * abs(a), losses
