"""Scaled token embedding on sm_100a kernels: ``out = scale * W[ids]`` (bf16), with the
backward scattering ``scale * d out`` into the fp32 ``main_grad`` of ``W`` (atomics)."""
from __future__ import annotations

import torch
from torch import Tensor

from .._native import cuda


class ScaledEmbedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids: Tensor, weight: Tensor, scale: float):
        ids = ids.to(torch.int32).contiguous().view(-1)
        out = torch.empty((ids.numel(), weight.shape[1]), dtype=torch.bfloat16, device=weight.device)
        cuda().embedding_fwd(ids, weight, out, scale)
        ctx.save_for_backward(ids)
        ctx.scale, ctx.weight = scale, weight
        return out

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        weight = ctx.weight
        main = getattr(weight, "main_grad", None)
        target = main if main is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        cuda().embedding_bwd(ids, dout.contiguous(), target, ctx.scale)
        return None, (None if main is not None else target.to(weight.dtype)), None


def scaled_embedding(ids: Tensor, weight: Tensor, scale: float) -> Tensor:
    if weight.dtype != torch.bfloat16:
        raise RuntimeError("the fused embedding runs on bf16 compute weights")
    out = ScaledEmbedding.apply(ids, weight, float(scale))
    return out.view(*ids.shape, weight.shape[1])
