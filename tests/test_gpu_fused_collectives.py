"""Multi-GPU (2 ranks, NCCL + symmetric memory): the fused-collective copy jobs on their own.

* gather: zeroed resident weights are refilled exactly from the owners' bf16 shards, by a job
  inside a GEMM (whose own output must not change) and by the standalone job kernel;
* push + ``shard_update``: a GEMM carrying the push of a finished fp32 gradient, then the
  step-end kernel, must leave every rank's master / moment / EMA / bf16 shards equal to an NCCL
  reduce-scatter of the same gradients followed by the AdamATan2 kernel, and a weight whose push
  did not run must be updated from its own (zero) rows without waiting.

Skipped with fewer than 2 GPUs."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, INTER = 256, 768


class _Block(torch.nn.Module):
    def __init__(self, dev):
        super().__init__()
        self.attn = torch.nn.Module()
        self.mlp = torch.nn.Module()
        self.attn.gqkv_proj = torch.nn.Module()
        self.attn.o_proj = torch.nn.Module()
        self.mlp.gate_up_proj = torch.nn.Module()
        self.mlp.down_proj = torch.nn.Module()
        g = torch.Generator(device="cpu").manual_seed(1)
        mk = lambda r, c: torch.nn.Parameter((torch.randn(r, c, generator=g) * 0.02).to(dev))  # noqa: E731
        self.attn.gqkv_proj.weight = mk(4 * H, H)
        self.attn.o_proj.weight = mk(H, H)
        self.mlp.gate_up_proj.weight = mk(2 * INTER, H)
        self.mlp.down_proj.weight = mk(H, INTER)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        from hrm_text_b200._native import cuda
        from hrm_text_b200.ops import gemm as G
        from hrm_text_b200.runtime.engine import ShardedParameters
        from hrm_text_b200.utils.errors import check_device_errors
        block = _Block(dev)
        P = ShardedParameters(block, beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99, fused=True)
        fc = P.fused
        slots = {s.fqn: s for s in P.slots}
        results = {}
        torch.manual_seed(100 + rank)
        cos = torch.rand(4096, 64, device=dev)
        sin = torch.rand(4096, 64, device=dev)
        # ---- gather: corrupt the resident copies, refill through GEMM-carried and standalone jobs
        M = 2048
        x = torch.randn(M, H, device=dev).bfloat16()
        res = torch.randn(M, H, device=dev).bfloat16()
        carrier_w = (torch.randn(H, H, device=dev) * 0.02).bfloat16()
        y_ref = G.linear(x, carrier_w, residual=res)
        w = {k: P.full_view(P.compute, s) for k, s in slots.items()}
        truth = {k: v.clone() for k, v in w.items()}
        for v in w.values():
            v.fill_(0)
        names = list(slots)
        for i, k in enumerate(names):
            if i % 2 == 0:  # inside a GEMM launch
                fc._gather_queue.append(fc.f1[k])
                y = G.linear(x, carrier_w, residual=res)
                assert torch.equal(y, y_ref), ("carrier GEMM output changed", k)
            else:
                fc._run_standalone(fc.f1[k], None)
        torch.cuda.synchronize()
        check_device_errors()
        for k in slots:
            assert torch.equal(w[k], truth[k]), ("gathered resident copy", k)
        # ---- F2: push + shard_update vs reduce-scatter + AdamATan2
        P.set_hyper(1e-3)
        state0 = {n: getattr(P, n).clone() for n in ("master", "exp_avg", "exp_avg_sq", "param_ema")}
        T = 1536
        grads_in = {}
        for k, s in slots.items():
            out_f, in_f = s.shape
            grads_in[k] = ((torch.randn(T, out_f, device=dev) * 1e-2).bfloat16(),
                           torch.randn(T, in_f, device=dev).bfloat16())
        # reference: local fp32 wgrads -> NCCL reduce-scatter -> AdamATan2 kernel on a copy of the state
        P.grad.zero_()
        for k, s in slots.items():
            dy, xx = grads_in[k]
            G.linear_wgrad_(dy, xx, P.full_view(P.grad, s))
        ref_shard = torch.zeros_like(P.master)
        for s in P.slots:
            dist.reduce_scatter_tensor(ref_shard[s.shard_off: s.shard_off + s.shard_numel],
                                       P.full_padded_view(P.grad, s))
        ref = {n: t.clone() for n, t in state0.items()}
        ref16 = torch.zeros(P.shard_numel, dtype=torch.bfloat16, device=dev)
        cuda().adam_atan2(ref["master"], ref_shard, ref["exp_avg"], ref["exp_avg_sq"], ref["param_ema"], ref16,
                          P.hyper, 0.9, 0.95, 0.1, 0.99)
        # fused: the gradients accumulated in main_grad in two parts (as the recurrent calls leave
        # them); pushes carried by a GEMM (first three weights) or run standalone (the last one)
        P.grad.zero_()
        fc.reset_step()
        dist.barrier()  # every rank's counts are zero before any push (the loss all-reduce in a step)
        for i, (k, s) in enumerate(slots.items()):
            dy, xx = grads_in[k]
            half = T // 2
            G.linear_wgrad_(dy[:half], xx[:half], P.full_view(P.grad, s))
            G.linear_wgrad_(dy[half:], xx[half:], P.full_view(P.grad, s))
            fc.queue_push(fc.f2[k])
            if i < 3:
                G.linear(x, carrier_w, residual=res)
        fc.flush()
        fc.update()
        torch.cuda.synchronize()
        check_device_errors()
        live = torch.zeros(P.shard_numel, dtype=torch.bool, device=dev)
        for s in P.slots:
            r0, r1 = s.local_rows(rank)
            live[s.shard_off: s.shard_off + (r1 - r0) * s.cols] = True
        for n in ("master", "exp_avg", "exp_avg_sq", "param_ema"):
            a, b = getattr(P, n)[live], ref[n][live]
            d = (a - b).abs()
            tol = 1e-6 + 1e-4 * b.abs()
            # fp32 atomics order differs between the two paths; atan2 of tiny moments can flip
            assert int((d > tol).sum()) <= max(2, a.numel() // 2000), (n, float(d.max()))
        d16 = (P.shard16[live].float() - ref16[live].float()).abs()
        assert int((d16 > 1e-2 * ref16[live].float().abs() + 1e-6).sum()) <= max(2, d16.numel() // 2000)
        # second step: the last weight has no gradient (its push never runs); its owner must not
        # wait for it and must update it from its own zero rows, as AdamATan2 with g = 0 does
        P.set_hyper(1e-3)
        names = list(slots)
        P.grad.zero_()
        for k in names[:3]:
            dy, xx = grads_in[k]
            G.linear_wgrad_(dy, xx, P.full_view(P.grad, slots[k]))
        ref_shard.zero_()
        for s in P.slots:
            dist.reduce_scatter_tensor(ref_shard[s.shard_off: s.shard_off + s.shard_numel],
                                       P.full_padded_view(P.grad, s))
        cuda().adam_atan2(ref["master"], ref_shard, ref["exp_avg"], ref["exp_avg_sq"], ref["param_ema"], ref16,
                          P.hyper, 0.9, 0.95, 0.1, 0.99)
        fc.reset_step()
        dist.barrier()
        for k in names[:3]:
            fc.queue_push(fc.f2[k])
        fc.flush()
        fc.update()
        torch.cuda.synchronize()
        check_device_errors()
        for n in ("master", "exp_avg", "exp_avg_sq", "param_ema"):
            a, b = getattr(P, n)[live], ref[n][live]
            d = (a - b).abs()
            assert int((d > 1e-6 + 1e-4 * b.abs()).sum()) <= max(2, a.numel() // 2000), ("step 2", n, float(d.max()))
        results["ok"] = True
        if rank == 0:
            torch.save(results, out)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_f1_f2_kernels_two_ranks(tmp_path):
    out = str(tmp_path / "r.pt")
    mp.spawn(_worker, args=(2, 29811, out), nprocs=2, join=True)
    assert torch.load(out)["ok"]
