"""RINS baseline (reference models/baselines/rins_nocarry.py:11-66).

Call plan: ``L_cycles`` calls of the L stack on ``"L"`` (starting at ``zL_init``) with the
embedded input ``"x"`` as injection, the last ``L_bp_cycles`` recording gradients, then one
H-stack call on the result without injection (always under the caller's grad mode). The
cache holds one slot per L call and a single H slot.

The stacks are ``Transformer`` subclasses themselves (``H_level.layers.*``), not wrapped in a
``core`` attribute as in HRM: those are the reference's parameter names for this family.
"""
from __future__ import annotations

from typing import Any, Optional

from torch import Tensor

from ..transformer import Transformer, TransformerConfig
from .recurrence import ModuleCall, PlannedRecurrence, init_state_vector, truncated


class RINSConfig(TransformerConfig):
    half_layers: bool = False
    L_cycles: int
    L_bp_cycles: int
    H_override: dict[str, Any] = {}


class RINSRecurrentBlock(Transformer):
    """A Transformer stack that is itself the level (``forward(hidden, injection)``)."""

    def forward(self, hidden_states: Tensor, input_injection: Optional[Tensor] = None, **kwargs) -> Tensor:  # type: ignore[override]
        return super().forward(hidden_states, injection=input_injection, **kwargs)


class RINS(PlannedRecurrence):
    output_state = "L"

    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = RINSConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be even when half_layers is set"
            config.n_layers //= 2
        self.H_level = RINSRecurrentBlock(TransformerConfig(**(config.model_dump() | config.H_override)))
        self.L_level = RINSRecurrentBlock(config)
        self.plan = [ModuleCall("L_level", "L", "x", ("L", i), g)
                     for i, g in enumerate(truncated(config.L_cycles, config.L_bp_cycles))]
        self.plan.append(ModuleCall("H_level", "L", None, ("H",), True))
        self.hidden_size = config.hidden_size
        self.head_hint = self.H_level.head_hint
        self.zL_init = init_state_vector(config.hidden_size)

    def call_plan(self) -> list[ModuleCall]:
        return self.plan

    def initial_states(self, x: Tensor) -> dict[str, Tensor]:
        return {"x": x, "L": self.zL_init}
