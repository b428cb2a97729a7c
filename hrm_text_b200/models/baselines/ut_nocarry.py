"""Universal Transformer baseline (reference models/baselines/ut_nocarry.py:12-49).

``cycles`` applications of one stack to ``z + x``, the last ``bp_cycles`` with grad.
"""
from __future__ import annotations

from contextlib import nullcontext
from typing import Optional

import torch
from torch import Tensor, nn

from ..common import trunc_normal_init_
from ..transformer import TransformerConfig
from .hrm_nocarry_bp_warmup import HierarchicalReasoningModelRecurrentBlock


class UniversalTransformerConfig(TransformerConfig):
    cycles: int
    bp_cycles: int


class UniversalTransformer(nn.Module):
    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = UniversalTransformerConfig(**config_dict)
        self.L_level = HierarchicalReasoningModelRecurrentBlock(TransformerConfig(**config.model_dump()))
        self.cycles, self.bp_cycles = config.cycles, config.bp_cycles
        self.head_hint = self.L_level.core.head_hint
        self.zL_init = nn.Buffer(trunc_normal_init_(torch.empty(config.hidden_size, dtype=torch.bfloat16), std=1.0),
                                 persistent=True)

    def create_cache(self, **kwargs):
        return [self.L_level.create_cache(**kwargs) for _ in range(self.cycles)]

    def forward(self, carry, x: Tensor, cache: Optional[list] = None, **seq_info):
        z = self.zL_init
        for i in range(self.cycles):
            ctx = nullcontext() if i >= self.cycles - self.bp_cycles else torch.no_grad()
            with ctx:
                z = self.L_level(z, x, cache=None if cache is None else cache[i], **seq_info)
        return None, z

    def compute_train_extra_args(self, train_state):
        return {}

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
