"""Token embedding, LM head, loss and training metrics (reference models/lm_head.py:18-74).

* Input: ``sqrt``-scaled embedding (``1/init_std`` with the backbone's input std).
* Output: untied ``lm_head`` Linear, then fp32 cross-entropy summed over tokens whose label
  is not ``IGNORE_LABEL_ID``.
* The loss is divided by the valid-token count averaged over data-parallel ranks
  (lm_head.py:52-55), so with a SUM gradient reduction every rank contributes as in a
  global mean.
* Metrics are ``(numerator, denominator)`` pairs: ``loss``, token ``accuracy`` and per-document
  ``exact_accuracy`` (lm_head.py:58-70).

On CUDA with labels, the head runs the fused kernel path
(``hrm_text_b200.ops.loss.lm_head_cross_entropy``): the lm_head GEMM epilogue emits per-tile
softmax statistics and argmax, so neither an fp32 copy of the logits nor a separate
softmax pass exists.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F
from pydantic import BaseModel
from torch import Tensor, nn

from .common import IGNORE_LABEL_ID, fused_path, segment_sum
from .layers import LinearInit, ScaledEmbeddingInit


class LMHeadConfig(BaseModel):
    vocab_size: int


def global_mean_count(count: Tensor) -> Tensor:
    """Mean of ``count`` over the default process group (identity without one)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        count = count.clone()
        dist.all_reduce(count, op=dist.ReduceOp.SUM)
        count = count / dist.get_world_size()
    return count


def training_metrics(loss_sum: Tensor, is_correct: Tensor, valid: Tensor, cu_seqlens: Tensor) -> dict:
    valid_count = valid.sum()
    seq_correct = segment_sum(is_correct.to(torch.int32), cu_seqlens)
    seq_valid = segment_sum(valid.to(torch.int32), cu_seqlens)
    seq_ok = seq_valid > 0
    return {
        "loss": (loss_sum.detach(), valid_count),
        "accuracy": (is_correct.sum(), valid_count),
        "exact_accuracy": (((seq_correct == seq_valid) & seq_ok).sum(), seq_ok.sum()),
    }


class LMHead(nn.Module):
    def __init__(self, model: nn.Module, config_dict: dict) -> None:
        super().__init__()
        self.model = model
        self.create_cache = self.model.create_cache
        self.compute_train_extra_args = self.model.compute_train_extra_args

        config = LMHeadConfig(**config_dict)
        hint = self.model.head_hint
        self.embed_tokens = ScaledEmbeddingInit(config.vocab_size, hint["in"]["dim"], init_std=hint["in"]["init_std"])
        self.lm_head = LinearInit(hint["out"]["dim"], config.vocab_size, bias=False, init_std=hint["out"]["init_std"])

    def embed(self, inputs: Tensor, dtype: torch.dtype) -> Tensor:
        if fused_path(inputs):
            from ..ops import embedding as emb_ops
            return emb_ops.scaled_embedding(inputs, self.embed_tokens.embedding_weight, self.embed_tokens.scale)
        return self.embed_tokens(inputs).to(dtype)

    def forward(self, carry, batch: dict, **kwargs) -> Tuple:
        weight = self.embed_tokens.embedding_weight
        compute_dtype = torch.bfloat16 if fused_path(weight) else weight.dtype
        hidden = self.embed(batch["inputs"], compute_dtype)
        passthrough = {k: v for k, v in batch.items() if k not in ("inputs", "labels")}
        if fused_path(hidden) and "cache" not in batch and "cu_seqlens" in batch:
            from ..ops.attention import PackedSeq
            passthrough["packed"] = PackedSeq(batch["position_ids"], batch["cu_seqlens"], batch["prefix_lens"])
        new_carry, hidden = self.model(carry, hidden, **passthrough, **kwargs)

        if "labels" not in batch:
            w = self.lm_head.weight
            if fused_path(hidden) and hidden.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 \
                    and w.shape[0] % 32 == 0:
                from ..ops import gemm as G  # tcgen05 GEMM (inference logits)
                flat = hidden.reshape(-1, hidden.shape[-1]).contiguous()
                return new_carry, G.infer_linear(flat, w).view(*hidden.shape[:-1], w.shape[0])
            return new_carry, F.linear(hidden, w.to(hidden.dtype))

        labels = batch["labels"]
        valid = labels != IGNORE_LABEL_ID
        if fused_path(hidden):
            from ..ops import loss as loss_ops
            loss_sum, is_correct = loss_ops.lm_head_cross_entropy(hidden, self.lm_head.weight, labels)
        else:
            logits = F.linear(hidden, self.lm_head.weight.to(hidden.dtype))
            loss_sum = F.cross_entropy(logits.float(), labels.long(), ignore_index=IGNORE_LABEL_ID, reduction="sum")
            with torch.no_grad():
                is_correct = torch.argmax(logits, dim=-1) == labels
        divisor = global_mean_count(valid.sum().to(torch.float32))
        with torch.no_grad():
            metrics = training_metrics(loss_sum, is_correct, valid, batch["cu_seqlens"])
        return new_carry, loss_sum / divisor, metrics
