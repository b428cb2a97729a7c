"""Small shared helpers of the model layer.

Parity notes (reference models/common.py):
* ``IGNORE_LABEL_ID`` is -100, the label that cross-entropy skips (common.py:7).
* ``trunc_normal_init_`` draws a normal truncated at 3 standard deviations and rescales it so
  the result has exactly the requested standard deviation (same distribution family and
  moments as common.py:10-13; computed here by inverse-CDF sampling plus an analytic
  variance correction).
* ``segment_sum`` plays the role of ``packing_sequence_sum`` (common.py:16-18): per-document
  sums over a packed token stream described by ``cu_seqlens``. Trailing zero padding in
  ``cu_seqlens`` yields non-positive entries, which callers treat as "no document".
* ``WrappedTensor`` keeps host-side scalar tensors away from device moves (common.py:21-32).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor

IGNORE_LABEL_ID = -100


def _truncated_std(bound: float) -> float:
    """Standard deviation of N(0,1) truncated to [-bound, bound]."""
    pdf = math.exp(-0.5 * bound * bound) / math.sqrt(2.0 * math.pi)
    mass = math.erf(bound / math.sqrt(2.0))
    return math.sqrt(1.0 - 2.0 * bound * pdf / mass)


_TRUNC3_STD = _truncated_std(3.0)


@torch.no_grad()
def trunc_normal_init_(tensor: Tensor, std: float = 1.0) -> Tensor:
    """Fill ``tensor`` with N(0, std^2) truncated at +-3 sigma (the sampled std is ``std``)."""
    if tensor.dtype in (torch.float32, torch.float64):
        torch.nn.init.trunc_normal_(tensor, mean=0.0, std=1.0, a=-3.0, b=3.0)
        return tensor.mul_(std / _TRUNC3_STD)
    tmp = torch.empty(tensor.shape, dtype=torch.float32, device=tensor.device)
    torch.nn.init.trunc_normal_(tmp, mean=0.0, std=1.0, a=-3.0, b=3.0)
    return tensor.copy_(tmp.mul_(std / _TRUNC3_STD))


def segment_sum(x: Tensor, cu_seqlens: Tensor) -> Tensor:
    """Sum of ``x`` over each segment ``[cu[i], cu[i+1])`` of a packed stream."""
    prefix = torch.zeros(x.shape[0] + 1, dtype=torch.int64 if not x.is_floating_point() else x.dtype,
                         device=x.device)
    torch.cumsum(x, dim=0, out=prefix[1:])
    cu = cu_seqlens.to(torch.int64)
    return prefix[cu[1:]] - prefix[cu[:-1]]


# The reference's name for the same operation.
packing_sequence_sum = segment_sum


@dataclass
class WrappedTensor:
    value: Tensor


def wrap_tensor(value: Tensor) -> WrappedTensor:
    return WrappedTensor(value)


def unwrap_tensor(value):
    return value.value if isinstance(value, WrappedTensor) else value


_FUSED_ENABLED = [True]


def fused_path(t) -> bool:
    """True when ``t`` lives on a GPU and the fused sm_100a path is enabled (the default)."""
    return bool(t.is_cuda and _FUSED_ENABLED[0])


class oracle_mode:
    """Context manager: run the plain-torch oracle path even on CUDA tensors (tests)."""

    def __enter__(self):
        self._prev = _FUSED_ENABLED[0]
        _FUSED_ENABLED[0] = False
        return self

    def __exit__(self, *exc):
        _FUSED_ENABLED[0] = self._prev
        return False
