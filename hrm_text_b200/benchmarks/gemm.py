"""GEMM microbenchmark over the HRM-Text layer shapes (tcgen05 kernel, fused epilogues).

    python -m hrm_text_b200.benchmarks.gemm [--size L|XL] [--tokens 21504] [--iters 20] [--only NAME]

Each case is timed with CUDA events over ``iters`` launches after warm-up; reports TFLOP/s.
Cases: the forward GEMMs of a layer (RoPE, SwiGLU, residual epilogues), their dgrad GEMMs
(SwiGLU-backward epilogue for the down projection), the fp32 weight-gradient GEMMs, and the
LM-head GEMM with the cross-entropy statistics epilogue (vocabulary 32768, logits not stored).
"""
from __future__ import annotations

import argparse
import json

import torch

SIZES = {"L": (1280, 3584, 10), "XL": (1536, 4096, 12), "B": (1024, 2816, 8)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", default="L", choices=sorted(SIZES))
    ap.add_argument("--tokens", type=int, default=21504)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", default=None)
    args = ap.parse_args(argv)
    from ..ops import gemm as G
    dev = torch.device("cuda", 0)
    h, inter, heads = SIZES[args.size]
    T = args.tokens
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).bfloat16()

    x = rnd(T, h)
    w_qkv, w_o, w_gu, w_d = rnd(4 * h, h, scale=0.03), rnd(h, h, scale=0.03), rnd(2 * inter, h, scale=0.03), \
        rnd(h, inter, scale=0.02)
    pos = torch.randint(0, 4096, (T,), device=dev, dtype=torch.int32)
    cos, sin = torch.rand(4096, 64, device=dev), torch.rand(4096, 64, device=dev)
    hmid = rnd(T, inter)
    gu = rnd(T, 2 * inter)
    dy_h = rnd(T, h, scale=0.01)
    dy_qkv = rnd(T, 4 * h, scale=0.01)
    grad_qkv = torch.zeros(4 * h, h, device=dev)
    grad_d = torch.zeros(h, inter, device=dev)
    grad_gu = torch.zeros(2 * inter, h, device=dev)
    grad_o = torch.zeros(h, h, device=dev)
    vocab = 32768
    w_head = rnd(vocab, h, scale=0.02)
    labels = torch.randint(0, vocab, (T,), device=dev, dtype=torch.int32)
    cases = {
        "qkv_rope": (lambda: G.linear_rope(x, w_qkv, pos, cos, sin, h, 3 * h), 2 * T * 4 * h * h),
        "o_residual": (lambda: G.linear(x, w_o, residual=x), 2 * T * h * h),
        "gate_up_swiglu": (lambda: G.linear_swiglu(x, w_gu), 2 * T * 2 * inter * h),
        "down_residual": (lambda: G.linear(hmid, w_d, residual=x), 2 * T * h * inter),
        "down_dgrad_swiglu": (lambda: G.linear_dgrad_swiglu(dy_h, w_d, gu), 2 * T * h * inter),
        "qkv_dgrad": (lambda: G.linear_dgrad(dy_qkv, w_qkv), 2 * T * 4 * h * h),
        "qkv_wgrad": (lambda: G.linear_wgrad_(dy_qkv, x, grad_qkv), 2 * T * 4 * h * h),
        "down_wgrad": (lambda: G.linear_wgrad_(dy_h, hmid, grad_d), 2 * T * h * inter),
        "gate_up_wgrad": (lambda: G.linear_wgrad_(gu, x, grad_gu), 2 * T * 2 * inter * h),
        "o_wgrad": (lambda: G.linear_wgrad_(dy_h, x, grad_o), 2 * T * h * h),
        "lm_head_ce": (lambda: G.lm_head_ce_stats(x, w_head, labels), 2 * T * vocab * h),
    }
    results = {}
    for name, (fn, flop) in cases.items():
        if args.only and name != args.only:
            continue
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        results[name] = {"ms": round(ms, 4), "tflops": round(flop / ms / 1e9, 1)}
    from ..utils.errors import check_device_errors
    check_device_errors()
    print(json.dumps({"size": args.size, "tokens": T, "cases": results}))


if __name__ == "__main__":
    main()
