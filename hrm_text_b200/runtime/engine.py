"""Training engine: in-house parameter sharding, fused optimizer, CUDA-graph step.

Replaces the reference's FSDP2 setup (pretrain.py:119-164, 206-212):

* **Sharding.** Every parameter is split along dim 0 into ``world`` chunks of
  ``ceil(rows / world)`` rows (the same chunking FSDP2 and DTensor ``Shard(0)`` use). A rank
  owns the fp32 master weights, ``exp_avg``, ``exp_avg_sq`` and EMA of its chunks only.
* **Resident compute weights.** The bf16 copies of all parameters live in one flat buffer
  that stays gathered for the whole step (forward through backward, across all 8
  recurrent module calls); module parameters are views into it.
* **Gradients.** fp32 gradient accumulators (one flat buffer, parameter-contiguous) are
  written directly by the weight-gradient GEMM epilogues (``param.main_grad``), then
  reduce-scattered with SUM (fp32, no division: the loss is pre-scaled by the global mean
  token count, lm_head.py:54-55, and AdamATan2 is scale-invariant).
* **Optimizer.** One fused AdamATan2 kernel over the flat local shard; it also writes the
  bf16 copy that the next step's all-gather distributes (or, on one GPU, the compute
  buffer directly).
* **Step capture.** ``GraphedTrainStep`` captures forward + backward + reduce-scatter +
  optimizer + all-gather in one CUDA graph per ``bp_steps`` value; per-step host inputs
  (batch, learning rate, bias corrections) are copied into static device buffers.

On CPU (tests, gloo) the same engine runs the torch oracle path in fp32.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor, nn

from ..optim.adam_atan2 import reference_update
from ..utils.trace import nvtx


@dataclass
class ParamSlot:
    fqn: str
    param: nn.Parameter
    shape: tuple
    rows: int
    cols: int
    chunk_rows: int
    full_off: int   # element offset in the full (padded) buffers
    shard_off: int  # element offset in the local shard buffers

    @property
    def numel(self) -> int:
        return self.rows * self.cols

    @property
    def full_padded(self) -> int:
        return self.chunk_rows * self.cols * self._world

    @property
    def shard_numel(self) -> int:
        return self.chunk_rows * self.cols

    _world: int = 1

    def local_rows(self, rank: int) -> tuple[int, int]:
        r0 = min(self.rows, rank * self.chunk_rows)
        return r0, min(self.rows, r0 + self.chunk_rows)


def _align(n: int, a: int = 64) -> int:
    return (n + a - 1) // a * a


class ShardedParameters:
    """Flat buffers for master shards, optimizer state, gradients and compute weights."""

    def __init__(self, model: nn.Module, *, beta1: float, beta2: float, weight_decay: float,
                 ema: Optional[float], group=None, compute_dtype: Optional[torch.dtype] = None,
                 fused: Optional[bool] = None):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        first = next(model.parameters())
        self.device = first.device
        self.on_cuda = first.is_cuda
        self.compute_dtype = compute_dtype or (torch.bfloat16 if self.on_cuda else torch.float32)
        self.beta1, self.beta2, self.weight_decay, self.ema = beta1, beta2, weight_decay, ema
        self.step_count = 0

        self.slots: list[ParamSlot] = []
        full_off = shard_off = 0
        for fqn, p in model.named_parameters():
            rows = p.shape[0] if p.dim() > 0 else 1
            cols = p.numel() // max(rows, 1)
            chunk = (rows + self.world - 1) // self.world
            slot = ParamSlot(fqn, p, tuple(p.shape), rows, cols, chunk, full_off, shard_off)
            slot._world = self.world
            self.slots.append(slot)
            full_off += _align(slot.full_padded)
            shard_off += _align(slot.shard_numel)
        self.full_numel, self.shard_numel = full_off, shard_off

        dev = self.device
        f32 = dict(dtype=torch.float32, device=dev)
        self.hyper = torch.zeros(4, **f32)  # lr, 1/bc1, 1/sqrt(bc2)
        if fused is None:
            # F1/F2 fused collectives (parallel/fused.py) are the default multi-GPU path;
            # HRM_FUSED_COLLECTIVES=0 selects the plain NCCL reduce-scatter / all-gather baseline
            fused = os.environ.get("HRM_FUSED_COLLECTIVES", "1") == "1"
        self.fused = None
        if fused and self.world > 1 and self.on_cuda:
            # F1/F2: optimizer state, gradient shard and bf16 shards in peer-addressable memory
            from ..parallel.fused import FusedCollectives
            self.fused = FusedCollectives(self, group)
            self.master = self.fused.view("master")
            self.exp_avg = self.fused.view("exp_avg") if beta1 > 0 else None
            self.exp_avg_sq = self.fused.view("exp_avg_sq")
            self.param_ema = self.fused.view("param_ema") if ema is not None else None
            self.grad_shard = self.fused.view("grad_shard")
            self.shard16 = self.fused.buf16
            self.grad = torch.zeros(self.full_numel, **f32)
        else:
            self.master = torch.zeros(self.shard_numel, **f32)
            self.exp_avg = torch.zeros(self.shard_numel, **f32) if beta1 > 0 else None
            self.exp_avg_sq = torch.zeros(self.shard_numel, **f32)
            self.param_ema = torch.zeros(self.shard_numel, **f32) if ema is not None else None
            self.grad = torch.zeros(self.full_numel, **f32)
            self.grad_shard = self.grad if self.world == 1 else torch.zeros(self.shard_numel, **f32)
            self.shard16 = None if self.world == 1 else torch.zeros(self.shard_numel, dtype=self.compute_dtype,
                                                                    device=dev)
        self.compute = torch.zeros(self.full_numel, dtype=self.compute_dtype, device=dev)

        with torch.no_grad():
            for s in self.slots:
                r0, r1 = s.local_rows(self.rank)
                flat = s.param.detach().reshape(s.rows, s.cols).float()
                self.master_view(s)[: (r1 - r0)].copy_(flat[r0:r1])
            if self.param_ema is not None:
                self.param_ema.copy_(self.master)
        self.gather_params()
        self._bind_module_params()

    # ------------------------------------------------------------------ views
    def master_view(self, s: ParamSlot) -> Tensor:
        return self.master[s.shard_off: s.shard_off + s.shard_numel].view(s.chunk_rows, s.cols)

    def shard_view(self, buf: Tensor, s: ParamSlot) -> Tensor:
        return buf[s.shard_off: s.shard_off + s.shard_numel].view(s.chunk_rows, s.cols)

    def full_view(self, buf: Tensor, s: ParamSlot) -> Tensor:
        return buf[s.full_off: s.full_off + s.numel].view(s.shape)

    def full_padded_view(self, buf: Tensor, s: ParamSlot) -> Tensor:
        return buf[s.full_off: s.full_off + s.full_padded]

    def _bind_module_params(self) -> None:
        for s in self.slots:
            s.param.data = self.full_view(self.compute, s)
            s.param.grad = None
            if self.on_cuda:
                s.param.main_grad = self.full_view(self.grad, s)
        if self.fused is not None:
            self.fused.attach()

    def _is_f1(self, s: ParamSlot) -> bool:
        return self.fused is not None and s.fqn in self.fused.f1

    def _is_f2(self, s: ParamSlot) -> bool:
        return self.fused is not None and s.fqn in self.fused.f2

    # ------------------------------------------------------------------ step pieces
    def zero_grad(self) -> None:
        self.grad.zero_()
        if self.fused is not None:
            self.fused.reset_step()
            for s in self.slots:
                if self._is_f2(s):
                    s.param._f2_pending = 0
        if not self.on_cuda:
            for s in self.slots:
                s.param.grad = None

    def collect_autograd_grads(self) -> None:
        """CPU path: move ``param.grad`` into the flat gradient buffer."""
        if self.on_cuda:
            return
        with torch.no_grad():
            for s in self.slots:
                if s.param.grad is not None:
                    self.full_view(self.grad, s).add_(s.param.grad.to(torch.float32))

    def reduce_grads(self) -> None:
        if self.world == 1:
            return
        if self.on_cuda:
            with dist._coalescing_manager(group=self.group, device=self.device):
                for s in self.slots:
                    if self._is_f2(s):
                        continue  # reduced (and updated) inside the fused wgrad kernel
                    dist.reduce_scatter_tensor(self.grad_shard[s.shard_off: s.shard_off + s.shard_numel],
                                               self.full_padded_view(self.grad, s), op=dist.ReduceOp.SUM,
                                               group=self.group)
        else:
            dist.all_reduce(self.grad, op=dist.ReduceOp.SUM, group=self.group)
            for s in self.slots:
                full = self.full_padded_view(self.grad, s).view(self.world, s.shard_numel)
                self.grad_shard[s.shard_off: s.shard_off + s.shard_numel].copy_(full[self.rank])

    def set_hyper(self, lr: float) -> None:
        """Advance the step counter and stage lr / bias corrections (host -> device)."""
        self.step_count += 1
        t = float(self.step_count)
        bc1 = 1.0 - self.beta1 ** t if self.beta1 > 0 else 1.0
        bc2 = 1.0 - self.beta2 ** t
        host = torch.tensor([lr, 1.0 / bc1, 1.0 / math.sqrt(bc2), t], dtype=torch.float32)
        if self.on_cuda:
            host = host.pin_memory()
        self.hyper.copy_(host, non_blocking=self.on_cuda)
        self._host_hyper = host  # keep the pinned source alive until the copy is done

    def optimizer_step(self) -> None:
        if self.on_cuda and self.fused is not None:
            self.fused.update()  # F2 inbox reduction + AdamATan2 for every local shard, one kernel
            return
        if self.on_cuda:
            from .._native import cuda
            out16 = self.compute if self.world == 1 else self.shard16
            cuda().adam_atan2(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, self.param_ema, out16,
                              self.hyper, self.beta1, self.beta2, self.weight_decay,
                              self.ema if self.ema is not None else 0.0)
            return
        lr = float(self.hyper[0])
        t = float(self.hyper[3])
        with torch.no_grad():
            reference_update(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, self.param_ema, t, lr,
                             self.beta1, self.beta2, self.weight_decay, self.ema)
            if self.world == 1:
                for s in self.slots:
                    self.full_view(self.compute, s).copy_(self.master_view(s).reshape(-1)[: s.numel].view(s.shape))
            else:
                self.shard16.copy_(self.master)

    def gather_params(self, all_slots: bool = False) -> None:
        """Distribute the updated bf16 shards to every rank's resident compute buffer.

        With fused collectives, F1 weights are gathered by their first GEMM of the next step
        instead (unless ``all_slots``); call ``sync_compute`` before using the model outside a
        training step.
        """
        if self.world == 1:
            if self.step_count == 0:  # initial fill
                with torch.no_grad():
                    for s in self.slots:
                        self.full_view(self.compute, s).copy_(
                            self.master_view(s).reshape(-1)[: s.numel].view(s.shape))
            return
        if self.step_count == 0:
            self.shard16.copy_(self.master)
            all_slots = True
        if self.on_cuda:
            with dist._coalescing_manager(group=self.group, device=self.device):
                for s in self.slots:
                    if not all_slots and self._is_f1(s):
                        continue
                    dist.all_gather_into_tensor(self.full_padded_view(self.compute, s),
                                                self.shard16[s.shard_off: s.shard_off + s.shard_numel],
                                                group=self.group)
        else:
            full = torch.zeros_like(self.compute)
            for s in self.slots:
                view = self.full_padded_view(full, s).view(self.world, s.shard_numel)
                view[self.rank].copy_(self.shard16[s.shard_off: s.shard_off + s.shard_numel])
            dist.all_reduce(full, op=dist.ReduceOp.SUM, group=self.group)
            self.compute.copy_(full)

    def sync_compute(self) -> None:
        """Bring the resident compute weights up to date outside a training step (the F1
        weights are otherwise gathered lazily by the next step's first GEMMs)."""
        if self.fused is not None and self.fused.f1:
            self.gather_params(all_slots=True)

    # ------------------------------------------------------------------ state access
    def full_param_fp32(self, s: ParamSlot, buf: Optional[Tensor] = None) -> Tensor:
        """Gather one parameter's fp32 tensor (from ``master`` or a state buffer) on every rank."""
        buf = self.master if buf is None else buf
        local = self.shard_view(buf, s).reshape(-1).contiguous()
        if self.world == 1:
            return local[: s.numel].view(s.shape).clone()
        out = torch.empty(self.world * s.shard_numel, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(out, local, group=self.group)
        return out[: s.numel].view(s.shape)

    def swap_ema(self) -> None:
        if self.param_ema is None:
            return
        tmp = self.master.clone()
        self.master.copy_(self.param_ema)
        self.param_ema.copy_(tmp)
        self.refresh_compute()

    def refresh_compute(self) -> None:
        """Re-derive the compute weights from the fp32 master shards."""
        if self.world == 1:
            with torch.no_grad():
                for s in self.slots:
                    self.full_view(self.compute, s).copy_(self.master_view(s).reshape(-1)[: s.numel].view(s.shape))
        else:
            self.shard16.copy_(self.master)
            self.gather_params(all_slots=True)


class TrainEngine:
    """One training step = forward, backward, gradient reduction, AdamATan2, parameter gather."""

    def __init__(self, model: nn.Module, *, beta1: float, beta2: float, weight_decay: float,
                 ema: Optional[float] = None, group=None):
        self.model = model
        self.params = ShardedParameters(model, beta1=beta1, beta2=beta2, weight_decay=weight_decay, ema=ema,
                                        group=group)
        self.carry = None

    def forward_backward(self, batch: dict, **extra):
        self.params.zero_grad()
        with nvtx("forward"):
            self.carry, loss, metrics = self.model(carry=self.carry, batch=batch, **extra)
        with nvtx("backward"):
            loss.backward()
        if self.params.fused is not None:
            self.params.fused.flush()  # gradient pushes that no backward GEMM carried
        self.params.collect_autograd_grads()
        return loss.detach(), metrics

    def step_body(self, batch: dict, **extra):
        loss, metrics = self.forward_backward(batch, **extra)
        with nvtx("reduce_grads"):
            self.params.reduce_grads()
        with nvtx("optimizer"):
            self.params.optimizer_step()
        with nvtx("gather"):
            self.params.gather_params()
        return loss, metrics

    def train_step(self, batch: dict, lr: float, **extra):
        self.params.set_hyper(lr)
        return self.step_body(batch, **extra)


BATCH_KEYS = ("inputs", "labels", "position_ids", "prefix_lens", "causal_lens", "cu_seqlens")


class GraphedTrainStep:
    """CUDA-graph capture of ``TrainEngine.step_body`` per ``bp_steps`` value.

    ``__call__(batch_host, lr, bp_steps)`` copies the (pinned) host batch into static device
    buffers, stages the optimizer scalars, and replays the captured step. It returns the
    static device tensors holding the loss and metrics of that step.
    """

    def __init__(self, engine: TrainEngine, example_batch: dict, warmup: int = 2):
        self.engine = engine
        dev = engine.params.device
        self.static = {k: torch.empty_like(example_batch[k], device=dev) for k in BATCH_KEYS}
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.outputs: dict[int, tuple] = {}
        self.pool = None
        self.warmup = warmup
        self.stream = torch.cuda.Stream(device=dev)

    def load(self, batch: dict) -> None:
        for k in BATCH_KEYS:
            self.static[k].copy_(batch[k], non_blocking=True)

    def capture(self, key, extra: dict) -> None:
        """Warm up eagerly (side stream), then capture one step body for ``extra`` kwargs."""
        eng = self.engine
        fused = eng.params.fused
        self.stream.wait_stream(torch.cuda.current_stream())
        if fused is not None:
            fused.set_f2_enabled(False)  # warm-up must not apply optimizer updates
        with torch.cuda.stream(self.stream):
            for _ in range(self.warmup):
                eng.forward_backward(self.static, **extra)
        if fused is not None:
            fused.set_f2_enabled(True)
        torch.cuda.current_stream().wait_stream(self.stream)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()  # release warm-up activations before the graph pool grows
        eng.params.zero_grad()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool, stream=self.stream, capture_error_mode="relaxed"):
            out = eng.step_body(self.static, **extra)
        self.pool = g.pool()
        self.graphs[key] = g
        self.outputs[key] = out

    def __call__(self, batch: dict, lr: float, bp_steps: int):
        self.load(batch)
        if bp_steps not in self.graphs:
            self.capture(bp_steps, {"bp_steps": bp_steps})  # warm-up runs forward/backward only
        self.engine.params.set_hyper(lr)
        self.graphs[bp_steps].replay()
        return self.outputs[bp_steps]

    def release(self) -> None:
        """Drop the graphs (required before destroying a process group they reference)."""
        self.graphs.clear()
        self.outputs.clear()
        self.pool = None
