"""PrefixLM attention microbenchmark.

    python -m hrm_text_b200.benchmarks.attention [--heads 16] [--tokens 21504] [--iters 20]
        [--kernel tcgen05|mma] [--only fwd|bwd|both] [--impl ours|reference]

bf16, head_dim 128, ``tokens`` packed tokens (documents log-normal, median 512, clipped to
[16, 4096], prefix fraction U[0, 0.5]), Q/K/V ~ N(0, 1) from seed 0. Each phase is timed
with CUDA events over ``iters`` launches after warm-up; reported with its useful FLOPs
(visible query-key pairs: 4 * pairs * 128 per head forward, 2.5x that backward).

``--impl reference`` times the reference's own op on the same packing and inputs:
``flash_attn_varlen_prefixlm`` from ``baseline/_ref/models/flash_attention_prefixlm_v2.py``
(two varlen passes, bidirectional prefix then causal response, models/flash_attention_prefixlm_v2.py:88-131
and :152-212) on the FlashAttention-2 stand-in for FA3 (``baseline/fa3_standin``). Its forward
excludes the sigmoid gate that ours fuses, and its backward excludes the gate and RoPE backward
that ours also does, so the comparison slightly favours the reference.
"""
from __future__ import annotations

import argparse
import json

import torch


def visible_pairs(cu, pl, n_docs) -> int:
    total = 0
    for i in range(n_docs):
        L = int(cu[i + 1] - cu[i])
        P = int(pl[i])
        total += P * P  # prefix queries see the whole prefix
        total += (L * (L + 1) - P * (P + 1)) // 2  # response query q sees keys [0, q]
    return total


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--tokens", type=int, default=21504)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--kernel", default="tcgen05", choices=["tcgen05", "mma"])
    ap.add_argument("--only", default="both", choices=["fwd", "bwd", "both"])
    ap.add_argument("--phases", action="store_true", help="trace the backward's per-phase cycles (tcgen05)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--noalloc", action="store_true",
                    help="also time the allocation-free C entry point (schedule build + forward per call)")
    args = ap.parse_args(argv)

    from ..data.synthetic import packed_batches
    from ..ops.attention import PackedSeq, attention_bwd, attention_fwd
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    T, H = args.tokens, args.heads
    b, s = next(iter(packed_batches(T, 32768, 4096, num_batches=1, seed=0)))
    packed = PackedSeq(b["position_ids"].to(dev), b["cu_seqlens"].to(dev), b["prefix_lens"].to(dev))
    sched = packed.schedule(False)
    qkv = torch.randn(T, 4 * H * 128, device=dev).bfloat16()
    pairs = visible_pairs(b["cu_seqlens"].tolist(), b["prefix_lens"].tolist(), s["numseqs"])
    fwd_flop = 4.0 * pairs * 128 * H
    cos = torch.ones(4096, 64, device=dev)
    sin = torch.zeros(4096, 64, device=dev)
    out = {"tokens": T, "heads": H, "docs": s["numseqs"], "visible_pairs": pairs, "kernel": args.kernel}

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.iters

    if args.impl == "reference":
        out.update(_reference_times(qkv, H, b, s, dev, timed, fwd_flop, args.only))
        out["kernel"] = "reference flash_attn_varlen_prefixlm on the FA3 stand-in"
        print(json.dumps(out))
        return

    o, y, lse = attention_fwd(qkv, H, sched, kernel=args.kernel)
    if args.only in ("fwd", "both"):
        ms = timed(lambda: attention_fwd(qkv, H, sched, kernel=args.kernel))
        out["fwd_ms"] = ms
        out["fwd_tflops"] = fwd_flop / ms / 1e9
    if args.noalloc:
        out.update(_noalloc_times(qkv, H, packed, timed, fwd_flop, o, y, lse))
    if args.only in ("bwd", "both"):
        dy = torch.randn(T, H * 128, device=dev).bfloat16()
        ms = timed(lambda: attention_bwd(qkv, H, sched, o, lse, dy, packed.position_ids, cos, sin))
        out["bwd_ms"] = ms
        out["bwd_tflops"] = 2.5 * fwd_flop / ms / 1e9
        if args.phases and args.kernel == "tcgen05":
            from ..ops.attention import bwd_phase_profile
            ph = bwd_phase_profile(lambda: attention_bwd(qkv, H, sched, o, lse, dy, packed.position_ids, cos, sin))
            blocks = max(1, ph.pop("query blocks"))
            out["bwd_phase_cycles_per_query_block"] = {k: round(v / blocks, 1) for k, v in ph.items()}
    from ..utils.errors import check_device_errors
    check_device_errors()
    print(json.dumps(out))


def _noalloc_times(qkv, H, packed, timed, fwd_flop, o, y, lse) -> dict:
    """``hrm_attn_fwd_noalloc`` through its exported C symbol, with the regular forward's schedule
    build included in the comparison (the entry point builds its schedule in every call)."""
    import ctypes

    import hrm_text_b200._C as ext
    from ..ops.attention import PackedSeq, attention_fwd
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.hrm_attn_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_void_p]
    T = qkv.shape[0]
    cu, pl = packed.cu_seqlens.to(torch.int32).contiguous(), packed.prefix_lens.to(torch.int32).contiguous()
    out, yy, ll = torch.empty_like(o), torch.empty_like(y), torch.empty_like(lse)

    def call():
        rc = fn(qkv.data_ptr(), qkv.stride(0), T, H, cu.data_ptr(), cu.numel(), pl.data_ptr(), 0, out.data_ptr(),
                yy.data_ptr(), out.stride(0), ll.data_ptr(), torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(f"hrm_attn_fwd_noalloc returned {rc}")

    ms = timed(call)
    ms_reg = timed(lambda: attention_fwd(qkv, H, PackedSeq(packed.position_ids, packed.cu_seqlens,
                                                            packed.prefix_lens).schedule(False)))
    return {"noalloc_fwd_ms": ms, "noalloc_fwd_tflops": fwd_flop / ms / 1e9,
            "regular_fwd_with_schedule_ms": ms_reg}


def _reference_times(qkv, H, b, s, dev, timed, fwd_flop, only) -> dict:
    """Forward / backward times of the reference's PrefixLM op on the same packed batch."""
    import os
    import sys
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    ref = os.path.join(root, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref, "models", "flash_attention_prefixlm_v2.py")):
        return {"unavailable": "baseline/_ref is missing"}
    sys.path.insert(0, os.path.join(root, "baseline", "fa3_standin"))
    sys.path.insert(0, ref)
    from models.flash_attention_prefixlm_v2 import flash_attn_varlen_prefixlm
    T = qkv.shape[0]
    w = H * 128
    q, k, v = (qkv[:, (i + 1) * w:(i + 2) * w].reshape(T, H, 128).contiguous().requires_grad_(True)
               for i in range(3))
    dtensors = {key: b[key].to(dev) for key in ("prefix_lens", "causal_lens", "cu_seqlens")}
    scalars = [torch.tensor(s[key]) for key in ("total_seqlen", "numseqs", "max_seqlen_prefix",
                                                "max_seqlen_causal", "max_seqlen_all")]

    def fwd():
        return flash_attn_varlen_prefixlm(q, k, v, False, dtensors["prefix_lens"], dtensors["causal_lens"],
                                          dtensors["cu_seqlens"], *scalars)
    res = {}
    if only in ("fwd", "both"):
        with torch.no_grad():
            ms = timed(fwd)
        res["fwd_ms"] = ms
        res["fwd_tflops"] = fwd_flop / ms / 1e9
    if only in ("bwd", "both"):
        o = fwd()
        dy = torch.randn(T, H, 128, device=dev).bfloat16()
        ms = timed(lambda: torch.autograd.grad(o, (q, k, v), dy, retain_graph=True))
        res["bwd_ms"] = ms
        res["bwd_tflops"] = 2.5 * fwd_flop / ms / 1e9
    return res


if __name__ == "__main__":
    main()
