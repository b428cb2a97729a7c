"""Tiny Recursive Model baseline (reference models/baselines/trm_nocarry.py:12-65).

The HRM recurrence with a single shared stack (``L_level``) used in both roles and fixed
per-level grad-call counts ``H_bp_steps`` / ``L_bp_steps``.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor, nn

from ..common import trunc_normal_init_
from ..transformer import TransformerConfig
from .hrm_nocarry_bp_warmup import HierarchicalReasoningModelRecurrentBlock


class TinyRecursiveModelConfig(TransformerConfig):
    half_layers: bool = False
    H_cycles: int
    L_cycles: int
    H_bp_steps: int
    L_bp_steps: int


class TinyRecursiveModel(nn.Module):
    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = TinyRecursiveModelConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be even when half_layers is set"
            config.n_layers //= 2
        self.L_level = HierarchicalReasoningModelRecurrentBlock(config)
        self.H_cycles, self.L_cycles = config.H_cycles, config.L_cycles
        self.H_bp_steps, self.L_bp_steps = config.H_bp_steps, config.L_bp_steps
        self.hidden_size = config.hidden_size
        self.head_hint = self.L_level.core.head_hint
        self.zL_init = nn.Buffer(trunc_normal_init_(torch.empty(config.hidden_size, dtype=torch.bfloat16), std=1.0),
                                 persistent=True)

    def create_cache(self, **kwargs):
        return dict(H=[self.L_level.create_cache(**kwargs) for _ in range(self.H_cycles)],
                    L=[self.L_level.create_cache(**kwargs) for _ in range(self.H_cycles * self.L_cycles)])

    def forward(self, carry, x: Tensor, cache: Optional[dict] = None, **seq_info):
        z_H, z_L = x, self.zL_init
        grad_on = torch.is_grad_enabled()
        n_l = self.H_cycles * self.L_cycles
        for i in range(self.H_cycles):
            for k in range(i * self.L_cycles, (i + 1) * self.L_cycles):
                with torch.set_grad_enabled(grad_on and k >= n_l - self.L_bp_steps):
                    z_L = self.L_level(z_L, z_H, cache=None if cache is None else cache["L"][k], **seq_info)
            with torch.set_grad_enabled(grad_on and i >= self.H_cycles - self.H_bp_steps):
                z_H = self.L_level(z_H, z_L, cache=None if cache is None else cache["H"][i], **seq_info)
        return None, z_H

    def compute_train_extra_args(self, train_state):
        return {}

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
