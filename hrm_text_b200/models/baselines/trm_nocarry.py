"""Tiny Recursive Model baseline (reference models/baselines/trm_nocarry.py:12-65).

TRM is the HRM call plan with one stack in both roles: ``recurrence.hierarchical_plan`` with
the high-level calls also routed to ``L_level``, and fixed per-role grad-call counts
(``H_bp_steps``, ``L_bp_steps``) instead of HRM's bp warm-up. The KV-cache layout keeps
separate H and L slots because the two roles see different hidden states.
"""
from __future__ import annotations

from torch import Tensor

from ..transformer import TransformerConfig
from .hrm_nocarry_bp_warmup import HierarchicalReasoningModelRecurrentBlock
from .recurrence import ModuleCall, PlannedRecurrence, hierarchical_plan, init_state_vector


class TinyRecursiveModelConfig(TransformerConfig):
    half_layers: bool = False
    H_cycles: int
    L_cycles: int
    H_bp_steps: int
    L_bp_steps: int


class TinyRecursiveModel(PlannedRecurrence):
    output_state = "H"

    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = TinyRecursiveModelConfig(**config_dict)
        if config.half_layers:
            assert config.n_layers % 2 == 0, "n_layers must be even when half_layers is set"
            config.n_layers //= 2
        self.L_level = HierarchicalReasoningModelRecurrentBlock(config)
        self.plan = hierarchical_plan(config.H_cycles, config.L_cycles, config.H_bp_steps, config.L_bp_steps,
                                      h_stack="L_level", l_stack="L_level")
        self.hidden_size = config.hidden_size
        self.head_hint = self.L_level.core.head_hint
        self.zL_init = init_state_vector(config.hidden_size)

    def call_plan(self) -> list[ModuleCall]:
        return self.plan

    def initial_states(self, x: Tensor) -> dict[str, Tensor]:
        return {"H": x, "L": self.zL_init}
