"""Hierarchical Reasoning Model with truncated backprop and a bp warm-up ramp.

Behaviour (reference models/baselines/hrm_nocarry_bp_warmup.py):
* two stacks, H and L, each with ``n_layers/2`` layers when ``half_layers`` (:46-53);
* state starts at ``z_H = x`` (the scaled embedding) and ``z_L = zL_init``, a bf16 ``[h]``
  buffer drawn from a unit truncated normal (:69, :76);
* ``H_cycles`` x (``L_cycles`` L-calls then one H-call); each call is
  ``stack(hidden + injection)`` with the other level's state as the injection (:34-43, :83-89);
* only the last ``bp_steps`` calls record gradients: H gets ``min(H_cycles, bp_steps-1)`` of
  them, L the rest (:78-81);
* ``bp_steps`` ramps linearly from ``bp_min_steps`` to ``bp_max_steps`` over the first
  ``bp_warmup_ratio`` of training (:93-97).

The recurrence is expressed as a call plan (``recurrence.hierarchical_plan``) that the shared
driver in ``recurrence.py`` runs.
"""
from __future__ import annotations

from typing import Any, Optional

from torch import Tensor, nn

from ..transformer import Transformer, TransformerConfig
from .recurrence import ModuleCall, PlannedRecurrence, hierarchical_plan, init_state_vector


class HierarchicalReasoningModelConfig(TransformerConfig):
    half_layers: bool = False

    H_cycles: int
    L_cycles: int

    bp_warmup_ratio: float = 0.0
    bp_min_steps: int = 2
    bp_max_steps: int = 5

    H_override: dict[str, Any] = {}


class HierarchicalReasoningModelRecurrentBlock(nn.Module):
    """One level: a Transformer stack applied to ``hidden + injection``."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.core = Transformer(config)
        self.create_cache = self.core.create_cache

    def forward(self, hidden_states: Tensor, input_injection: Optional[Tensor], **kwargs) -> Tensor:
        return self.core(hidden_states, injection=input_injection, **kwargs)


def split_bp_steps(bp_steps: int, h_cycles: int) -> tuple[int, int]:
    """(H grad calls, L grad calls): H first, L keeps at least one."""
    h_bp = min(h_cycles, bp_steps - 1)
    return h_bp, bp_steps - h_bp


def bp_steps_schedule(step: int, total_steps: int, warmup_ratio: float, lo: int, hi: int) -> int:
    warmup = total_steps * warmup_ratio
    progress = min(1.0, step / warmup) if warmup > 0 else 1.0
    return lo + int(progress * (hi - lo))


class HierarchicalReasoningModel(PlannedRecurrence):
    output_state = "H"
    plan_kwargs = ("bp_steps",)

    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = HierarchicalReasoningModelConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be even when half_layers is set"
            config.n_layers //= 2
        self.config = config

        self.H_level = HierarchicalReasoningModelRecurrentBlock(
            TransformerConfig(**(config.model_dump() | config.H_override)))
        self.L_level = HierarchicalReasoningModelRecurrentBlock(config)

        self.H_cycles, self.L_cycles = config.H_cycles, config.L_cycles
        self.bp_warmup_ratio = config.bp_warmup_ratio
        self.bp_min_steps, self.bp_max_steps = config.bp_min_steps, config.bp_max_steps
        self.hidden_size = config.hidden_size
        self.head_hint = self.H_level.core.head_hint
        self.zL_init = init_state_vector(config.hidden_size)

    def call_plan(self, bp_steps: int = 2) -> list[ModuleCall]:
        """The module calls of one forward, in order (``bp_steps`` of them record gradients)."""
        h_bp, l_bp = split_bp_steps(bp_steps, self.H_cycles)
        return hierarchical_plan(self.H_cycles, self.L_cycles, h_bp, l_bp)

    def initial_states(self, x: Tensor) -> dict[str, Tensor]:
        return {"H": x, "L": self.zL_init}

    def compute_train_extra_args(self, train_state: Any) -> dict[str, Any]:
        return dict(bp_steps=bp_steps_schedule(train_state.step, train_state.total_steps, self.bp_warmup_ratio,
                                               self.bp_min_steps, self.bp_max_steps))
