"""AdamATan2: AdamW with ``atan2(m, sqrt(v))`` in place of ``m / (sqrt(v) + eps)``.

Update rule per parameter (reference models/adam_atan2.py:60-97), with ``t`` the step count:

    p  <- p * (1 - lr * wd)                               (decoupled weight decay)
    m  <- m + (1 - b1) * (g - m)                          (skipped when b1 == 0)
    v  <- b2 * v + (1 - b2) * g^2
    p  <- p - lr / (1 - b1^t) * atan2(m, sqrt(v) / sqrt(1 - b2^t))
                       (no momentum: p <- p - lr * atan2(g, sqrt(v) / sqrt(1 - b2^t)))
    ema <- ema + (1 - ema_decay) * (p - ema)              (when ema_decay is set)

State keys are ``step`` (0-d fp32 tensor), ``exp_avg``, ``exp_avg_sq`` and ``param_ema`` so
``torch.distributed.checkpoint.state_dict.get_optimizer_state_dict`` produces the layout the
reference writes and reads.

``step()`` here is the torch implementation (CPU oracle and small models). The training
engine updates parameters with the fused CUDA kernel (``hrm_text_b200.ops.optim``) that
implements the same rule on fp32 master shards; ``reference_update`` below is the
per-tensor formula both are tested against.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor
from torch.optim.optimizer import Optimizer


@torch.no_grad()
def reference_update(param: Tensor, grad: Tensor, exp_avg: Optional[Tensor], exp_avg_sq: Tensor,
                     param_ema: Optional[Tensor], step: float, lr: float, beta1: float, beta2: float,
                     weight_decay: float, ema: Optional[float]) -> None:
    """One AdamATan2 update of a single tensor in fp32 (``step`` is the new step count)."""
    if weight_decay != 0:
        param.mul_(1.0 - lr * weight_decay)
    if exp_avg is not None:
        exp_avg.lerp_(grad, 1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1.0 - beta2)
    bc1 = 1.0 - beta1 ** step
    bc2_sqrt = (1.0 - beta2 ** step) ** 0.5
    denom = exp_avg_sq.sqrt() / bc2_sqrt
    if exp_avg is not None:
        param.add_(torch.atan2(exp_avg, denom), alpha=-lr / bc1)
    else:
        param.add_(torch.atan2(grad, denom), alpha=-lr)
    if param_ema is not None and ema is not None:
        param_ema.lerp_(param, 1.0 - ema)


class AdamATan2(Optimizer):
    def __init__(self, params, lr: float | Tensor = 1e-3, betas: Tuple[float, float] = (0.9, 0.95),
                 weight_decay: float = 0.1, ema: Optional[float] = None):
        if isinstance(lr, Tensor) and lr.numel() != 1:
            raise ValueError("Tensor lr must have one element")
        if not 0.0 <= float(lr):
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta1: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta2: {betas[1]}")
        if not 0.0 <= weight_decay:
            raise ValueError(f"Invalid weight_decay: {weight_decay}")
        super().__init__(params, dict(lr=lr, betas=betas, weight_decay=weight_decay, ema=ema))
        self._init_state()

    @torch.no_grad()
    def _init_state(self) -> None:
        for group in self.param_groups:
            for p in group["params"]:
                state = self.state[p]
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                if group["betas"][0] > 0:
                    state["exp_avg"] = torch.zeros_like(p)
                state["exp_avg_sq"] = torch.zeros_like(p)
                if group["ema"] is not None:
                    state["param_ema"] = p.detach().clone()

    @torch.no_grad()
    def step(self, closure=None):  # type: ignore[override]
        assert closure is None, "closures are not supported"
        for group in self.param_groups:
            lr = float(group["lr"])
            beta1, beta2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                state = self.state[p]
                state["step"] += 1
                reference_update(p, p.grad, state.get("exp_avg"), state["exp_avg_sq"], state.get("param_ema"),
                                 float(state["step"]), lr, beta1, beta2, group["weight_decay"], group["ema"])

    @torch.no_grad()
    def swap_ema(self) -> None:
        """Exchange parameters and their EMA (call again to swap back)."""
        for group in self.param_groups:
            for p in group["params"]:
                state = self.state[p]
                if "param_ema" in state:
                    tmp = p.detach().clone()
                    p.copy_(state["param_ema"])
                    state["param_ema"].copy_(tmp)
