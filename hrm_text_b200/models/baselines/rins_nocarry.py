"""RINS baseline (reference models/baselines/rins_nocarry.py:11-66).

``L_cycles`` applications of the L stack to ``z_L + x`` (the last ``L_bp_cycles`` with grad),
then one H-stack call on the final ``z_L`` without injection.
"""
from __future__ import annotations

from contextlib import nullcontext
from typing import Any, Optional

import torch
from torch import Tensor, nn

from ..common import trunc_normal_init_
from ..transformer import Transformer, TransformerConfig


class RINSConfig(TransformerConfig):
    half_layers: bool = False
    L_cycles: int
    L_bp_cycles: int
    H_override: dict[str, Any] = {}


class RINSRecurrentBlock(Transformer):
    """A Transformer stack that is itself the level (keeps the reference's FQNs: ``H_level.layers``)."""

    def forward(self, hidden_states: Tensor, input_injection: Optional[Tensor] = None, **kwargs) -> Tensor:  # type: ignore[override]
        return super().forward(hidden_states, injection=input_injection, **kwargs)


class RINS(nn.Module):
    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = RINSConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be even when half_layers is set"
            config.n_layers //= 2
        self.H_level = RINSRecurrentBlock(TransformerConfig(**(config.model_dump() | config.H_override)))
        self.L_level = RINSRecurrentBlock(config)
        self.L_cycles, self.L_bp_cycles = config.L_cycles, config.L_bp_cycles
        self.hidden_size = config.hidden_size
        self.head_hint = self.H_level.head_hint
        self.zL_init = nn.Buffer(trunc_normal_init_(torch.empty(config.hidden_size, dtype=torch.bfloat16), std=1.0),
                                 persistent=True)

    def create_cache(self, **kwargs):
        return dict(H=self.H_level.create_cache(**kwargs),
                    L=[self.L_level.create_cache(**kwargs) for _ in range(self.L_cycles)])

    def forward(self, carry, x: Tensor, cache: Optional[dict] = None, **seq_info):
        z_L = self.zL_init
        for i in range(self.L_cycles):
            ctx = nullcontext() if i >= self.L_cycles - self.L_bp_cycles else torch.no_grad()
            with ctx:
                z_L = self.L_level(z_L, x, cache=None if cache is None else cache["L"][i], **seq_info)
        return None, self.H_level(z_L, None, cache=None if cache is None else cache["H"], **seq_info)

    def compute_train_extra_args(self, train_state):
        return {}

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
