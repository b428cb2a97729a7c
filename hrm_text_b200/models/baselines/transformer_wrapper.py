"""Plain Transformer adapted to the carry protocol (reference models/baselines/transformer_wrapper.py:6-17)."""
from __future__ import annotations

import torch
from torch import Tensor

from ..transformer import Transformer, TransformerConfig


class TransformerWrapper(Transformer):
    def __init__(self, config_dict: dict) -> None:
        super().__init__(TransformerConfig(**config_dict))

    def forward(self, carry, x: Tensor, **kwargs):  # type: ignore[override]
        return None, super().forward(x, **kwargs)

    def compute_train_extra_args(self, train_state):
        return {}

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
