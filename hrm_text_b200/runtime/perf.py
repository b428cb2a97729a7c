"""Training throughput accounting: model FLOPs per step, device-timed tokens/s and MFU.

The reference logs only loss / accuracy / lr (pretrain.py:366-370). The training loop here
adds, at every log interval:

* ``perf/tokens_per_s`` — whole-job tokens per second over the interval, from CUDA events
  recorded on the training stream after each step; the interval's device time is the
  maximum over ranks (one all-reduce of a float, issued by every rank at the same point);
* ``perf/step_ms`` — that device time per step;
* ``perf/tflops_per_gpu`` and ``perf/mfu`` — model FLOPs (linear layers of every module call
  the call plan runs, the LM head, and attention over the step's actual packing) per second
  per GPU, and that as a fraction of the bf16 dense peak (``HRM_PEAK_TFLOPS``, default 2250).

FLOPs count a multiply-add as 2. Forward-only calls count 2 FLOPs per weight per token;
grad-enabled calls add 4 for the backward (data and weight gradients). Attention counts the
visible (query, key) pairs of every document: 4·pairs·hidden forward, 10·pairs·hidden backward.
"""
from __future__ import annotations

import os
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist


def _stack_params(stack) -> int:
    return sum(p.numel() for p in stack.parameters())


def _attention_pairs(cu_seqlens: np.ndarray, prefix_lens: np.ndarray, causal: bool) -> int:
    """Visible (query, key) pairs of one packing (key j visible to query i iff j < max(P, i+1))."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    n = int(np.argmax(cu[1:] <= cu[:-1])) if np.any(cu[1:] <= cu[:-1]) else len(cu) - 1
    lens = cu[1:n + 1] - cu[:n]
    p = np.zeros_like(lens) if causal else np.minimum(np.asarray(prefix_lens[:n], dtype=np.int64), lens)
    return int((p * p + (lens * (lens + 1) - p * (p + 1)) // 2).sum())


def step_flops(model, batch: dict, extra: Optional[dict] = None) -> float:
    """Model FLOPs of one training step of ``model`` (an ``LMHead``) on one rank's ``batch``."""
    extra = extra or {}
    core = model.model
    tokens = int(batch["inputs"].numel())
    flops = 0.0
    calls = []
    if hasattr(core, "call_plan"):
        plan = core.call_plan(**{k: v for k, v in extra.items() if k in getattr(core, "plan_kwargs", ())})
        calls = [(getattr(core, c.stack), c.grad) for c in plan]
    else:  # a single stack applied once with gradients (plain Transformer)
        calls = [(core, True)]
    cu = batch.get("cu_seqlens")
    pairs = 0
    if cu is not None:
        pl = batch.get("prefix_lens")
        pl = pl.cpu().numpy() if pl is not None else np.zeros(len(cu))
        pairs = _attention_pairs(cu.cpu().numpy(), pl, False)
    for stack, grad in calls:
        cfg = getattr(stack, "config", None) or getattr(getattr(stack, "core", None), "config", None)
        params = _stack_params(stack)
        flops += (2 + (4 if grad else 0)) * params * tokens
        if cfg is not None:
            flops += (4 + (10 if grad else 0)) * pairs * cfg.hidden_size * cfg.n_layers
    head = model.lm_head.weight.numel()
    flops += 6 * head * tokens
    return flops


class ThroughputMeter:
    """Device-timed throughput over log intervals (see the module docstring)."""

    def __init__(self, device: torch.device, world: int = 1, peak_tflops: Optional[float] = None):
        self.device = device
        self.world = world
        self.peak = 1e12 * (peak_tflops if peak_tflops is not None else float(os.environ.get("HRM_PEAK_TFLOPS",
                                                                                               "2250")))
        self.cuda = device.type == "cuda"
        self._start = None
        self._t0 = None
        self._steps = 0
        self._tokens = 0
        self._flops = 0.0

    def begin(self) -> None:
        """Mark the start of an interval (call before the interval's first step is launched)."""
        if self.cuda:
            self._start = torch.cuda.Event(enable_timing=True)
            self._start.record()
        else:
            import time
            self._t0 = time.perf_counter()
        self._steps, self._tokens, self._flops = 0, 0, 0.0

    def step(self, tokens_global: int, flops_local: float) -> None:
        if self._start is None and self._t0 is None:
            self.begin()
        self._steps += 1
        self._tokens += tokens_global
        self._flops += flops_local

    def report(self) -> dict:
        """Close the interval (every rank must call this at the same point) and start the next."""
        if self._steps == 0:
            return {}
        if self.cuda:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            end.synchronize()
            seconds = self._start.elapsed_time(end) / 1000.0
        else:
            import time
            seconds = time.perf_counter() - self._t0
        if dist.is_initialized():
            t = torch.tensor([seconds], dtype=torch.float64, device=self.device if self.cuda else "cpu")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            seconds = float(t.item())
        out = {"perf/tokens_per_s": self._tokens / seconds, "perf/step_ms": 1000.0 * seconds / self._steps,
               "perf/tflops_per_gpu": self._flops / seconds / 1e12, "perf/mfu": self._flops / seconds / self.peak}
        self.begin()
        return out
