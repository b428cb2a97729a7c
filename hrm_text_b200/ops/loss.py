"""Fused LM head + cross-entropy on sm_100a kernels; the ``[T, V]`` logits are never stored.

Forward: one tcgen05 GEMM over the whole vocabulary whose epilogue reduces each 128-column
slice of every logit row to softmax statistics (row max, sum of exponentials, argmax and, when
the label falls in the slice, the label's logit) without writing the logits anywhere; a small
kernel combines the partials into the log-sum-exp, the per-row fp32 loss and token
correctness. The reference materialises the bf16 logits and an fp32 copy for
``F.cross_entropy`` (models/lm_head.py:43-55).

Backward, one vocabulary chunk of ``chunk`` rows of the head at a time (default 8192,
``HRM_CE_CHUNK``): a GEMM recomputes the chunk's logits and its epilogue turns them into
``(softmax - onehot) * dloss`` (bf16, zero for rows without a label) using the forward's
log-sum-exp; a dgrad GEMM adds ``dlogits_c @ W_c`` into an fp32 ``d hidden`` accumulator and
an fp32 wgrad GEMM adds ``dlogits_c^T @ hidden`` into rows ``c`` of the head weight's
``main_grad``. Only one ``[T, chunk]`` bf16 buffer exists at a time.
"""
from __future__ import annotations

import os

import torch
from torch import Tensor

from .._native import cuda
from . import gemm as G

DEFAULT_CHUNK = int(os.environ.get("HRM_CE_CHUNK", "8192"))


class LMHeadCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden: Tensor, weight: Tensor, labels: Tensor, chunk: int):
        labels = labels.to(torch.int32).contiguous()
        hidden = hidden.contiguous()
        pmax, psum, parg, tgt = G.lm_head_ce_stats(hidden, weight, labels)
        T = hidden.shape[0]
        lse = torch.empty((T,), dtype=torch.float32, device=hidden.device)
        loss_rows = torch.empty((T,), dtype=torch.float32, device=hidden.device)
        correct = torch.empty((T,), dtype=torch.uint8, device=hidden.device)
        cuda().ce_finalize(pmax, psum, parg, tgt, labels, lse, loss_rows, correct)
        ctx.save_for_backward(hidden, weight, lse, labels)
        ctx.chunk = chunk
        ctx.mark_non_differentiable(correct)
        return loss_rows.sum(), correct

    @staticmethod
    def backward(ctx, grad_loss, _grad_correct):
        hidden, weight, lse, labels = ctx.saved_tensors
        grad = grad_loss.detach().to(torch.float32).reshape(1).contiguous()
        T, H = hidden.shape
        V = weight.shape[0]
        chunk = min(ctx.chunk, V)
        d32 = torch.zeros((T, H), dtype=torch.float32, device=hidden.device)
        main = getattr(weight, "main_grad", None)
        g_w = main if main is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        dl = torch.empty((T, chunk), dtype=torch.bfloat16, device=hidden.device)
        for c0 in range(0, V, chunk):
            c1 = min(V, c0 + chunk)
            w_c = weight[c0:c1]
            dl_c = dl[:, : c1 - c0]
            G.lm_head_ce_dlogits(hidden, w_c, labels, lse, grad, c0, dl_c)
            G.linear_dgrad_accumulate_(dl_c, w_c, d32)
            G.linear_wgrad_(dl_c, hidden, g_w[c0:c1])
        d_hidden = torch.empty((T, H), dtype=torch.bfloat16, device=hidden.device)
        cuda().cast_f32_bf16(d32, d_hidden)
        return d_hidden, (None if main is not None else g_w.to(weight.dtype)), None, None


def lm_head_cross_entropy(hidden: Tensor, weight: Tensor, labels: Tensor,
                          chunk: int = DEFAULT_CHUNK) -> tuple[Tensor, Tensor]:
    """Returns ``(sum of per-token CE over valid labels (fp32), is_correct (bool [T]))``."""
    if weight.dtype != torch.bfloat16:
        raise RuntimeError("the fused LM head runs on bf16 compute weights (engine / model.to(torch.bfloat16))")
    if chunk % 256 != 0:
        raise ValueError("the vocabulary chunk must be a multiple of 256")
    loss_sum, correct = LMHeadCrossEntropy.apply(hidden, weight, labels, chunk)
    return loss_sum, correct.bool()
