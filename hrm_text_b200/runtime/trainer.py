"""Public training API.

``Trainer`` is what a user (and ``pretrain.py``) calls: build a model from an arch config,
wrap it in the sharded engine, and run steps from host batches::

    trainer = Trainer(model_cfg, lr_betas..., device=torch.device("cuda", local_rank))
    loss = trainer.train_step(host_batch, lr=2.5e-4, bp_steps=5)   # float

``train_step`` copies the step's (pinned) host batch to the device, runs the captured
CUDA graph for this ``bp_steps`` (forward, backward, gradient reduce-scatter, AdamATan2,
parameter all-gather) and reads the loss back. ``train_step_async`` skips the read-back
and returns device tensors (loss, metrics).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from .engine import BATCH_KEYS, GraphedTrainStep, TrainEngine
from .factory import build_model


class Trainer:
    def __init__(self, model_cfg: dict, *, beta1: float = 0.9, beta2: float = 0.95, weight_decay: float = 0.1,
                 ema: Optional[float] = None, device: Optional[torch.device] = None, group=None,
                 use_cuda_graphs: bool = True, model: Optional[nn.Module] = None):
        self.device = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                                 else torch.device("cpu"))
        self.model = model if model is not None else build_model(model_cfg, self.device)
        self.engine = TrainEngine(self.model, beta1=beta1, beta2=beta2, weight_decay=weight_decay, ema=ema,
                                  group=group)
        self.use_graphs = use_cuda_graphs and self.device.type == "cuda"
        self._graphed: Optional[GraphedTrainStep] = None

    @property
    def params(self):
        return self.engine.params

    def _to_device(self, batch: dict) -> dict:
        return {k: batch[k].to(self.device, non_blocking=True) for k in BATCH_KEYS}

    def train_step_async(self, batch: dict, lr: float, bp_steps: Optional[int] = None):
        extra = {} if bp_steps is None else {"bp_steps": bp_steps}
        if self.use_graphs:
            if self._graphed is None:
                self._graphed = GraphedTrainStep(self.engine, batch)
            key = -1 if bp_steps is None else bp_steps
            return self._graphed_call(batch, lr, key, extra)
        return self.engine.train_step(self._to_device(batch), lr, **extra)

    def _graphed_call(self, batch, lr, key, extra):
        g = self._graphed
        g.load(batch)
        if key not in g.graphs:
            g.capture(key, extra)
        self.engine.params.set_hyper(lr)
        g.graphs[key].replay()
        return g.outputs[key]

    def train_step(self, batch: dict, lr: float, bp_steps: Optional[int] = None) -> float:
        loss, _ = self.train_step_async(batch, lr, bp_steps)
        return float(loss.item())

    def sync_weights(self) -> None:
        """Make ``self.model``'s weights current for use outside ``train_step`` (inference,
        evaluation). On several GPUs the block weights are gathered lazily by the next step's
        first GEMMs, so between steps the resident copies of those weights lag one update."""
        self.engine.params.sync_compute()

    def close(self) -> None:
        if self._graphed is not None:
            self._graphed.release()
            self._graphed = None
