"""Fused LM head + cross-entropy on sm_100a kernels.

Forward: one tcgen05 GEMM whose epilogue writes the bf16 logits and, per 256-column tile,
the row max, sum of exponentials, argmax and (when the label falls in the tile) the label's
logit; a small kernel combines the partials into log-sum-exp, per-row fp32 loss and token
correctness. There is no fp32 copy of the logits and no separate softmax pass (the
reference upcasts the full ``[T, V]`` logits to fp32 for ``F.cross_entropy``,
models/lm_head.py:52).

Backward: the bf16 logits are turned into ``(softmax - onehot) * dloss`` in place, then a
dgrad GEMM gives ``d hidden`` and an fp32 wgrad GEMM accumulates into the head weight's
``main_grad``.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .._native import cuda
from . import gemm as G


class LMHeadCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden: Tensor, weight: Tensor, labels: Tensor):
        labels = labels.to(torch.int32).contiguous()
        hidden = hidden.contiguous()
        logits, pmax, psum, parg, tgt = G.lm_head_ce_logits(hidden, weight, labels)
        T = hidden.shape[0]
        lse = torch.empty((T,), dtype=torch.float32, device=hidden.device)
        loss_rows = torch.empty((T,), dtype=torch.float32, device=hidden.device)
        correct = torch.empty((T,), dtype=torch.uint8, device=hidden.device)
        cuda().ce_finalize(pmax, psum, parg, tgt, labels, lse, loss_rows, correct)
        ctx.save_for_backward(hidden, weight, logits, lse, labels)
        ctx.mark_non_differentiable(correct)
        return loss_rows.sum(), correct

    @staticmethod
    def backward(ctx, grad_loss, _grad_correct):
        hidden, weight, logits, lse, labels = ctx.saved_tensors
        grad = grad_loss.detach().to(torch.float32).reshape(1).contiguous()
        cuda().ce_dlogits(logits, lse, labels, grad)  # logits now hold dlogits
        d_hidden = G.linear_dgrad(logits, weight)
        main = getattr(weight, "main_grad", None)
        if main is not None:
            G.linear_wgrad_(logits, hidden, main)
            d_weight = None
        else:
            g = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
            G.linear_wgrad_(logits, hidden, g)
            d_weight = g.to(weight.dtype)
        return d_hidden, d_weight, None


def lm_head_cross_entropy(hidden: Tensor, weight: Tensor, labels: Tensor) -> tuple[Tensor, Tensor]:
    """Returns ``(sum of per-token CE over valid labels (fp32), is_correct (bool [T]))``."""
    if weight.dtype != torch.bfloat16:
        raise RuntimeError("the fused LM head runs on bf16 compute weights (engine / model.to(torch.bfloat16))")
    loss_sum, correct = LMHeadCrossEntropy.apply(hidden, weight, labels)
    return loss_sum, correct.bool()
