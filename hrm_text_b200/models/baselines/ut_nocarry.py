"""Universal Transformer baseline (reference models/baselines/ut_nocarry.py:12-49).

Call plan: ``cycles`` calls of one stack on the state ``"z"`` (starting at ``zL_init``) with
the embedded input ``"x"`` as injection; the last ``bp_cycles`` record gradients. The cache is
a list with one slot per call.
"""
from __future__ import annotations

from torch import Tensor

from ..transformer import TransformerConfig
from .hrm_nocarry_bp_warmup import HierarchicalReasoningModelRecurrentBlock
from .recurrence import ModuleCall, PlannedRecurrence, init_state_vector, truncated


class UniversalTransformerConfig(TransformerConfig):
    cycles: int
    bp_cycles: int


class UniversalTransformer(PlannedRecurrence):
    output_state = "z"

    def __init__(self, config_dict: dict) -> None:
        super().__init__()
        config = UniversalTransformerConfig(**config_dict)
        self.L_level = HierarchicalReasoningModelRecurrentBlock(TransformerConfig(**config.model_dump()))
        self.plan = [ModuleCall("L_level", "z", "x", (i,), g)
                     for i, g in enumerate(truncated(config.cycles, config.bp_cycles))]
        self.head_hint = self.L_level.core.head_hint
        self.zL_init = init_state_vector(config.hidden_size)

    def call_plan(self) -> list[ModuleCall]:
        return self.plan

    def initial_states(self, x: Tensor) -> dict[str, Tensor]:
        return {"x": x, "z": self.zL_init}
