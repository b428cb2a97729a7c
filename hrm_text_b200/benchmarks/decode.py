"""Batched decode throughput (inference): generated tokens per second of one decode step over
``batch`` sequences with ``context`` cached tokens each, HRM-Text L or XL, bf16, 1 GPU.

    python -m hrm_text_b200.benchmarks.decode [--size L|XL] [--batch 32] [--context 512]
        [--steps 50] [--impl ours|reference]

Both arms build the model with random-init weights, fill every slot's KV caches with random
keys / values up to ``context`` tokens (decode cost does not depend on the values) and time
``steps`` decode steps with CUDA events after warm-up; the cache lengths advance by one per
step as in generation. ``ours`` replays the CUDA graph that ``generate_tokens`` uses
(``inference.engine.DecodeGraph``: fused kernels, no library GEMM). ``reference`` calls the
reference's own ``_batched_decode`` (``torch.compile(dynamic=False, fullgraph=True)``,
simple_inference_engine.py:110-112) on the reference model, with its KV-cache attention
(``flash_attn_with_kvcache``) served by the FlashAttention-2 stand-in for FA3.
Reported: decode tokens/s = batch * steps / time (sampling excluded in both arms).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

VOCAB, MAX_SEQ_LEN = 32768, 4096


def _fill(cache, context: int) -> None:
    for leaf in torch.utils._pytree.tree_leaves(cache):
        if isinstance(leaf, torch.Tensor):
            leaf[:, :context].normal_()


def _timed(fn, steps: int, warmup: int, lengths: torch.Tensor) -> float:
    start = lengths.clone()
    for _ in range(warmup):
        fn()
        lengths.add_(1)
    lengths.copy_(start)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
        lengths.add_(1)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_ours(args) -> dict:
    from ..inference.engine import DecodeGraph
    from ..runtime.factory import arch_preset, build_model
    dev = torch.device("cuda", 0)
    cfg = arch_preset("hrm", args.size) | dict(vocab_size=VOCAB, max_seq_len=MAX_SEQ_LEN)
    torch.manual_seed(0)
    model = build_model(cfg, dev).to(torch.bfloat16).eval()
    max_tokens = args.context + args.steps + args.warmup + 8
    cache = model.create_cache(max_batch_size=args.batch, max_seq_len=max_tokens, dtype=torch.bfloat16, device=dev)
    with torch.inference_mode():
        graph = DecodeGraph(model, None, cache, args.batch, dev)
        _fill(cache, args.context)
        tokens = torch.randint(0, VOCAB, (args.batch,), device=dev)
        lengths = torch.full((args.batch,), args.context, dtype=torch.int32, device=dev)
        ms = _timed(lambda: graph(tokens, lengths), args.steps, args.warmup, lengths)
    return {"impl": "ours", "ms_per_step": ms}


def _import_with_py313_generator(name: str):
    """Import a reference module whose annotations use Python 3.13's two-argument
    ``typing.Generator[Y, S]`` (the reference targets 3.13; this interpreter is 3.12): while it
    is imported, ``typing.Generator`` accepts two arguments and fills in the default return
    type ``None``. Only annotation objects are affected, not the module's computation."""
    import importlib
    import typing
    original = typing.Generator

    class _GeneratorAlias:
        def __getitem__(self, item):
            item = item if isinstance(item, tuple) else (item,)
            return original[item + (None,) * (3 - len(item))]

        def __getattr__(self, name):  # everything else is typing.Generator's
            return getattr(original, name)

    typing.Generator = _GeneratorAlias()
    try:
        return importlib.import_module(name)
    finally:
        typing.Generator = original


def run_reference(args) -> dict:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    ref = os.path.join(root, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref, "simple_inference_engine.py")):
        return {"impl": "reference", "unavailable": "baseline/_ref is missing"}
    sys.path.insert(0, root)
    from baseline.reference_arm import _install_import_shims, ref_arch
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"  # Inductor's CPU codegen needs an OpenMP-capable g++
    _install_import_shims()
    sie = _import_with_py313_generator("simple_inference_engine")  # the reference's module
    from utils.functions import load_model_class
    arch = ref_arch(args.size)
    cfg = arch | {"vocab_size": VOCAB, "max_seq_len": MAX_SEQ_LEN}
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = load_model_class(arch["head"])(load_model_class(arch["name"])(cfg), cfg)
    model = model.to(torch.bfloat16).eval()
    max_tokens = args.context + args.steps + args.warmup + 8
    cache = model.create_cache(max_batch_size=args.batch, max_seq_len=max_tokens, dtype=torch.bfloat16, device="cuda")
    with torch.inference_mode():
        _fill(cache, args.context)
        tokens = torch.randint(0, VOCAB, (args.batch,), device="cuda")
        lengths = torch.full((args.batch,), args.context, dtype=torch.int32, device="cuda")
        ms = _timed(lambda: sie._batched_decode(model, None, tokens, cache, lengths), args.steps, args.warmup, lengths)
    return {"impl": "reference", "ms_per_step": ms}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", default="L", choices=["L", "XL"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--context", type=int, default=512)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args(argv)
    out = run_ours(args) if args.impl == "ours" else run_reference(args)
    out.update(size=args.size, batch=args.batch, context=args.context, steps=args.steps)
    if "ms_per_step" in out:
        out["decode_tokens_per_s"] = args.batch / (out["ms_per_step"] / 1000.0)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
