"""NVTX ranges for timeline profilers (Nsight Systems, ``ncu --nvtx``).

Ranges mark every module call of the recurrence (``L_level[L,3] grad``), every kernel family
of the fused block (``gemm.gqkv_rope``, ``attention.fwd``, ``rmsnorm.bwd``, ...) and the
engine's step phases (``forward_backward``, ``reduce_grads``, ``optimizer``, ``gather``).
They are off unless ``HRM_NVTX=1``: a disabled range is one shared no-op context manager.
Inside a captured CUDA graph the ranges mark the capture, not the replays.
"""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("HRM_NVTX", "0") == "1"
_NOOP = contextlib.nullcontext()


def nvtx(name: str):
    """``with nvtx("attention.fwd"): ...`` — a profiler range when enabled, else a no-op."""
    if not ENABLED:
        return _NOOP
    return torch.cuda.nvtx.range(name)


def set_enabled(flag: bool) -> None:
    global ENABLED
    ENABLED = bool(flag)
