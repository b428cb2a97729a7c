"""Recurrence as data: one driver runs every recurrent model family's forward.

HRM, TRM, RINS and UT all apply one or two Transformer stacks repeatedly to a few named
states, each application being ``state <- stack(state + injection)`` with gradients recorded
only for the last few applications (truncated backprop). Here a model does not spell out
loops; it *describes* one forward as a call plan, an ordered list of :class:`ModuleCall`:

* ``stack``  — the submodule to run (``"H_level"`` or ``"L_level"``);
* ``state``  — the state it reads and overwrites;
* ``inject`` — the state added to it as the input injection (``None``: no injection);
* ``slot``   — where the call's KV cache lives in the cache structure (inference);
* ``grad``   — whether the call records gradients.

:func:`run_plan` executes a plan, :func:`cache_for_plan` allocates the cache structure a
plan addresses, and :class:`PlannedRecurrence` is the ``nn.Module`` base that ties them to
the carry protocol every architecture in this package follows
(``forward(carry, x, cache=None, **seq_info) -> (carry, hidden)``).

A cache ``slot`` is a short tuple: ``("L", 3)`` means ``cache["L"][3]``, ``("H",)`` means
``cache["H"]`` and ``(2,)`` means ``cache[2]``; the cache layouts (and so every checkpoint-free
inference path) stay those of the reference models.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Optional

import torch
from torch import Tensor, nn

from ...utils.trace import nvtx
from ..common import trunc_normal_init_


@dataclass(frozen=True)
class ModuleCall:
    stack: str
    state: str
    inject: Optional[str]
    slot: tuple
    grad: bool


def truncated(n_calls: int, n_grad: int) -> list[bool]:
    """Grad flags of ``n_calls`` consecutive calls of which the last ``n_grad`` record gradients."""
    return [i >= n_calls - n_grad for i in range(n_calls)]


def hierarchical_plan(h_cycles: int, l_cycles: int, h_grad: int, l_grad: int, h_stack: str = "H_level",
                      l_stack: str = "L_level") -> list[ModuleCall]:
    """``h_cycles`` x (``l_cycles`` low-level calls, then one high-level call).

    The low level updates ``"L"`` with ``"H"`` as injection and the high level the reverse;
    the last ``l_grad`` low-level and last ``h_grad`` high-level calls record gradients.
    """
    l_flags = truncated(h_cycles * l_cycles, l_grad)
    h_flags = truncated(h_cycles, h_grad)
    plan = []
    for i in range(h_cycles):
        for k in range(i * l_cycles, (i + 1) * l_cycles):
            plan.append(ModuleCall(l_stack, "L", "H", ("L", k), l_flags[k]))
        plan.append(ModuleCall(h_stack, "H", "L", ("H", i), h_flags[i]))
    return plan


def lookup(cache: Any, slot: tuple) -> Any:
    if cache is None:
        return None
    for key in slot:
        cache = cache[key]
    return cache


def cache_for_plan(plan: list[ModuleCall], make: Callable[[str], Any]) -> Any:
    """Allocate one cache per distinct slot of ``plan`` (``make(stack)`` creates one)."""
    slots: dict[tuple, str] = {}
    for call in plan:
        slots.setdefault(call.slot, call.stack)
    if all(len(s) == 1 and isinstance(s[0], int) for s in slots):
        return [make(slots[(i,)]) for i in range(len(slots))]
    out: dict[str, Any] = {}
    for slot, stack in slots.items():
        if len(slot) == 1:
            out[slot[0]] = make(stack)
        else:
            out.setdefault(slot[0], {})[slot[1]] = make(stack)
    return {k: [v[i] for i in range(len(v))] if isinstance(v, dict) else v for k, v in out.items()}


def run_plan(model: nn.Module, plan: list[ModuleCall], states: dict[str, Tensor], cache: Any = None,
             **seq_info) -> dict[str, Tensor]:
    """Execute ``plan`` on ``states`` (updated in place and returned)."""
    grad_on = torch.is_grad_enabled()
    for call in plan:
        stack = getattr(model, call.stack)
        with nvtx(f"{call.stack}{list(call.slot)}{' grad' if call.grad else ''}"), \
                torch.set_grad_enabled(grad_on and call.grad):
            states[call.state] = stack(states[call.state], None if call.inject is None else states[call.inject],
                                       cache=lookup(cache, call.slot), **seq_info)
    return states


def init_state_vector(hidden_size: int) -> nn.Buffer:
    """The learned-at-init ``[h]`` bf16 start state (unit truncated normal), broadcast over tokens."""
    return nn.Buffer(trunc_normal_init_(torch.empty(hidden_size, dtype=torch.bfloat16), std=1.0), persistent=True)


class PlannedRecurrence(nn.Module):
    """Base for models whose forward is a call plan.

    Subclasses define ``call_plan(**plan_kwargs)``, ``initial_states(x)`` and ``output_state``;
    ``plan_kwargs`` names the forward keyword arguments that shape the plan (e.g. ``bp_steps``).
    """

    output_state: str = "H"
    plan_kwargs: tuple[str, ...] = ()

    def call_plan(self, **kwargs) -> list[ModuleCall]:
        raise NotImplementedError

    def initial_states(self, x: Tensor) -> dict[str, Tensor]:
        raise NotImplementedError

    def forward(self, carry, x: Tensor, cache: Any = None, **kwargs):
        plan_args = {k: kwargs.pop(k) for k in self.plan_kwargs if k in kwargs}
        states = run_plan(self, self.call_plan(**plan_args), self.initial_states(x), cache, **kwargs)
        return None, states[self.output_state]

    def create_cache(self, **kwargs):
        return cache_for_plan(self.call_plan(), lambda stack: getattr(self, stack).create_cache(**kwargs))

    def compute_train_extra_args(self, train_state: Any) -> dict[str, Any]:
        return {}

    def initial_carry(self, batch_size: int, dtype: torch.dtype) -> None:
        return None
