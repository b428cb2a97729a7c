"""Fused-collective sweep, run with one process per GPU:

    torchrun --nproc-per-node N -m hrm_text_b200.benchmarks.fused [--size XL] [--tokens 4096,16384,32768]

At the size preset's layer shapes, for each token count M per GPU, with the QKV GEMM (RoPE
epilogue, M x 4h x h) as the carrier kernel:
  (a) param-shard all-gather of the down-projection weight (h x inter, bf16):
        fused  the QKV GEMM carrying the gather job (peer loads by its epilogue warps)
        base   the same GEMM + NCCL all_gather_into_tensor of the bf16 shard
  (b) down-projection gradient reduce-scatter + AdamATan2 shard update:
        fused  the QKV GEMM carrying the push job (peer stores + counts) + the step-end
               shard_update kernel for that weight (+ the counter reset and the tiny all-reduce
               that orders it before the peers' pushes, which a training step gets from its
               loss all-reduce)
        base   the same GEMM + NCCL reduce_scatter_tensor (fp32) + AdamATan2 kernel
``carrier_ms`` is the GEMM alone. Times are CUDA-event device times, max over ranks.
Roofline = max(carrier FLOPs / measured bf16 peak, bytes that must cross NVLink / 770 GB/s per
direction); ``frac`` = roofline / achieved. Weights N(0, 0.02), activations N(0, 1),
gradients N(0, 1e-3).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist
from torch import nn

SIZES = {"L": (1280, 3584), "XL": (1536, 4096)}
NVLINK_GBS = 770.0     # measured peer copy bandwidth per direction (B200 pool)


def _peak_tflops() -> float:
    """Measured cuBLAS bf16 burst throughput (MEASURED_PEAKS.json next to the repository), else
    the earlier measurement on the same pool."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


PEAK_TFLOPS = _peak_tflops()


class _Layer(nn.Module):
    """Parameter names that the engine's F1/F2 selection recognises."""

    def __init__(self, h, inter, dev):
        super().__init__()
        self.attn = nn.Module()
        self.mlp = nn.Module()
        self.attn.gqkv_proj = nn.Module()
        self.mlp.down_proj = nn.Module()
        self.attn.gqkv_proj.weight = nn.Parameter(torch.randn(4 * h, h, device=dev) * 0.02)
        self.mlp.down_proj.weight = nn.Parameter(torch.randn(h, inter, device=dev) * 0.02)


def _time(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", default="XL", choices=sorted(SIZES))
    ap.add_argument("--tokens", default="4096,16384,32768")
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()

    from ..ops import gemm as G
    from ..runtime.engine import ShardedParameters
    h, inter = SIZES[args.size]
    torch.manual_seed(0)
    layer = _Layer(h, inter, dev)
    params = ShardedParameters(layer, beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.9999, fused=True)
    params.set_hyper(2.2e-4)
    slots = {s.fqn: s for s in params.slots}
    s_qkv, s_down = slots["attn.gqkv_proj.weight"], slots["mlp.down_proj.weight"]
    w_qkv, w_down = layer.attn.gqkv_proj.weight, layer.mlp.down_proj.weight
    fc = params.fused
    g_down = fc.f1[s_down.fqn]
    p_down = fc.f2[s_down.fqn]
    down_items = fc._work_items(only=s_down.fqn)
    sync_word = torch.zeros(1, device=dev)
    cos = torch.rand(4096, 64, device=dev)
    sin = torch.rand(4096, 64, device=dev)
    results = []
    for M in [int(x) for x in args.tokens.split(",")]:
        x = torch.randn(M, h, device=dev).bfloat16()
        pos = torch.randint(0, 4096, (M,), device=dev, dtype=torch.int32)
        shard_d = params.shard16[s_down.shard_off: s_down.shard_off + s_down.shard_numel]
        full_d = params.full_padded_view(params.compute, s_down)
        w_down.main_grad.copy_(torch.randn_like(w_down.main_grad) * 1e-3)
        grad_sl = slice(s_down.shard_off, s_down.shard_off + s_down.shard_numel)

        def carrier():
            G.linear_rope(x, w_qkv, pos, cos, sin, h, 3 * h)

        def fused_a():
            fc._gather_queue.append(g_down)
            carrier()

        def base_a():
            carrier()
            dist.all_gather_into_tensor(full_d, shard_d)

        def fused_b():
            fc.reset_step()
            dist.all_reduce(sync_word)
            fc.queue_push(p_down)
            carrier()
            fc.update(down_items)  # owner: wait for the pushes, sum, AdamATan2

        def base_b():
            from .._native import cuda
            carrier()
            dist.reduce_scatter_tensor(params.grad_shard[grad_sl], params.full_padded_view(params.grad, s_down))
            cuda().adam_atan2(params.master[grad_sl], params.grad_shard[grad_sl], params.exp_avg[grad_sl],
                              params.exp_avg_sq[grad_sl], params.param_ema[grad_sl], params.shard16[grad_sl],
                              params.hyper, 0.9, 0.95, 0.1, 0.9999)

        t_c = _time(carrier, args.iters)
        ta_f, ta_b = _time(fused_a, args.iters), _time(base_a, args.iters)
        tb_f, tb_b = _time(fused_b, args.iters), _time(base_b, args.iters)
        fc.reset_step()
        dist.barrier()
        flop = 2.0 * M * 4 * h * h
        bytes_a = (world - 1) / world * h * inter * 2
        bytes_b = (world - 1) / world * h * inter * 4
        roof_a = max(flop / PEAK_TFLOPS / 1e9, bytes_a / NVLINK_GBS / 1e6)
        roof_b = max(flop / PEAK_TFLOPS / 1e9, bytes_b / NVLINK_GBS / 1e6)
        results.append({"tokens": M, "carrier_ms": t_c,
                        "a_allgather_down": {"fused_ms": ta_f, "baseline_ms": ta_b, "roofline_ms": roof_a,
                                             "fused_frac": roof_a / ta_f, "baseline_frac": roof_a / ta_b},
                        "b_rs_adam_down": {"fused_ms": tb_f, "baseline_ms": tb_b, "roofline_ms": roof_b,
                                           "fused_frac": roof_b / tb_f, "baseline_frac": roof_b / tb_b}})
    from ..utils.errors import check_device_errors
    check_device_errors()
    if rank == 0:
        print(json.dumps({"size": args.size, "world": world, "results": results}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
