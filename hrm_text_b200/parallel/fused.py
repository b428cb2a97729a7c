"""Fused collectives of the sharding engine (multi-GPU, CUDA): peer memory and copy jobs.

Replaces the two FSDP2 collectives of the reference step (pretrain.py:119-128, the per-block
parameter all-gather; :150-155, the fp32 SUM gradient reduce-scatter) for the four weights of
every Transformer block (``gqkv_proj``, ``o_proj``, ``gate_up_proj``, ``down_proj``). The bf16
shards and the fp32 optimizer state / gradient inbox live in symmetric buffers, so every rank
can address every other rank's copy over NVLink. The transfers are copy jobs
(csrc/kernels/collective_jobs.cuh) that ride inside the GEMM kernels the step launches anyway:
the epilogue warps of every CTA run them before their first tile, overlapping the GEMM's math.

* **F1 — all-gather.** The step's first-use order of the block weights is recorded on the
  first step. From then on, the first weight is gathered by a standalone job kernel at the start
  of the step, and every later weight by a job inside the GEMM launched just before its first
  use (one gather per GEMM launch, in first-use order), so the consuming GEMM reads its weight
  from local memory in its normal tile order. The resident copy serves every later call of
  the step (the recurrent cycles, the backward): each weight byte crosses NVLink once per step.
* **F2 — reduce-scatter.** The step's last weight-gradient GEMM of a weight accumulates into
  the local fp32 gradient as every other one does; the next GEMM launched then carries a push
  job that stores the rows other ranks own into this rank's slot of each owner's inbox and
  counts every 32 x 128 region there. Pushes that no GEMM took by the end of the backward run
  as a standalone job kernel. At the end of the step one kernel per rank (``shard_update``)
  waits for its counts, sums its own rows and the peers' slots in rank order, and runs
  AdamATan2 + EMA on its shards, writing the bf16 shard the next step gathers.

The embedding, LM head and norm weights stay on NCCL (reduce-scatter before ``shard_update``,
all-gather after it). Cross-rank ordering comes from collectives every step already has:
* the loss-divisor all-reduce at the end of the forward separates every rank's reset of its
  counts (``reset_step``) and its gathers from peer shards from any peer's pushes and
  ``shard_update`` writes of that step;
* the step-end NCCL all-gather separates every rank's ``shard_update`` (bf16 shards written,
  inbox read) from the next step's gathers and pushes.
"""
from __future__ import annotations

import os
from collections import deque
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

BLOCK_WEIGHTS = ("attn.gqkv_proj.weight", "attn.o_proj.weight", "mlp.gate_up_proj.weight", "mlp.down_proj.weight")
ITEM_ELEMS = 1 << 16  # elements per shard_update work item for NCCL-reduced parameters


@dataclass
class F1Info:
    fqn: str
    src: torch.Tensor        # device int64 [world]: address of each rank's bf16 shard of the weight
    dst: torch.Tensor        # the local resident copy (the module parameter's data)
    chunk_rows: int
    owner: "FusedCollectives" = field(repr=False, default=None)
    pending: bool = False    # set at the start of a step, cleared at the weight's first use


@dataclass
class F2Info:
    fqn: str
    src: torch.Tensor        # the local fp32 gradient of the weight (main_grad)
    inbox_off: int           # fp32 elements from the symmetric base: this weight in inbox slot 0
    cnt_off: int             # int32 elements from the symmetric base: the owner's 32-row counts
    chunk_rows: int
    ran_index: int           # element of the local count buffer set when the push ran this step
    owner: "FusedCollectives" = field(repr=False, default=None)
    enabled: bool = True


def f2_eligible(rows: int, cols: int, chunk_rows: int) -> bool:
    return rows % 32 == 0 and cols % 32 == 0 and chunk_rows % 32 == 0


def f1_eligible(cols: int) -> bool:
    return cols % 8 == 0  # 16-byte rows


class FusedCollectives:
    """Symmetric buffers, counters and per-weight F1 / F2 metadata for one ``ShardedParameters``."""

    def __init__(self, params, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        self.params = params
        self.group = group or dist.group.WORLD
        self.world, self.rank = params.world, params.rank
        dev = params.device
        S = params.shard_numel
        names = ["master", "exp_avg", "exp_avg_sq", "param_ema", "grad_shard"]
        self.region = {n: i * S for i, n in enumerate(names)}
        self.region["inbox"] = len(names) * S  # [world][S]: one slot per source rank

        enable_f1 = os.environ.get("HRM_F1", "1") != "0"
        enable_f2 = os.environ.get("HRM_F2", "1") != "0"
        block = [s for s in params.slots if s.fqn.endswith(BLOCK_WEIGHTS)]
        f1_slots = [s for s in block if enable_f1 and f1_eligible(s.cols)]
        f2_slots = [s for s in block if enable_f2 and f2_eligible(s.rows, s.cols, s.chunk_rows)]

        cnt_sizes = {s.fqn: s.chunk_rows // 32 for s in f2_slots}
        self.cnt_off = (len(names) + self.world) * S
        n32 = self.cnt_off + ((sum(cnt_sizes.values()) + 63) // 64) * 64
        self.buf32 = symm_mem.empty(n32, dtype=torch.float32, device=dev)
        self.handle32 = symm_mem.rendezvous(self.buf32, self.group)
        self.buf16 = symm_mem.empty(S, dtype=torch.bfloat16, device=dev)
        self.handle16 = symm_mem.rendezvous(self.buf16, self.group)
        self.buf32.zero_()
        self.buf16.zero_()
        self.base32 = torch.tensor(list(self.handle32.buffer_ptrs), dtype=torch.int64, device=dev)

        # local per-step flags: one per F2 weight, set by its push job (one memset per step)
        self.local_counts = torch.zeros(max(1, len(f2_slots)), dtype=torch.int32, device=dev)
        self.f1: dict[str, F1Info] = {}
        self.f2: dict[str, F2Info] = {}
        cnt = self.cnt_off
        for i, s in enumerate(f2_slots):
            self.f2[s.fqn] = F2Info(s.fqn, None, self.region["inbox"] + s.shard_off, cnt, s.chunk_rows, i, owner=self)
            cnt += cnt_sizes[s.fqn]
        for s in f1_slots:
            src = torch.tensor([int(b) + s.shard_off * 2 for b in self.handle16.buffer_ptrs], dtype=torch.int64,
                               device=dev)
            self.f1[s.fqn] = F1Info(s.fqn, src, None, s.chunk_rows, owner=self)
        self.counters = self.buf32[self.cnt_off:].view(torch.int32)
        self.items = self._work_items()
        # copy-job scheduling (host side, per step)
        self.order: Optional[list] = None   # first-use order of the F1 weights (recorded on the first step)
        self._recording: list = []
        self._gather_queue: deque = deque()
        self._push_queue: deque = deque()
        self._gathered: set = set()
        self._desc_cache: dict = {}

    def _work_items(self, only: Optional[str] = None) -> torch.Tensor:
        """``shard_update`` work list: 32-row groups of F2 weights (wait on their counts, sum the
        inbox), fixed-size pieces of every other parameter (gradient from the NCCL reduce-scatter).
        An F2 item also names its weight's push flag: the kernel skips the wait and the inbox when
        the weight's push did not run this step (no gradient through it: every rank runs the same
        recurrence schedule, so no rank pushed). ``only``: the items of one
        parameter (benchmarks)."""
        p = self.params
        rows = []
        for s in p.slots:
            if only is not None and s.fqn != only:
                continue
            if s.fqn in self.f2:
                info = self.f2[s.fqn]
                r0, r1 = s.local_rows(self.rank)
                expected = (self.world - 1) * -(-s.cols // 128)
                for g in range((r1 - r0) // 32):
                        rows.append((s.shard_off + g * 32 * s.cols, 32 * s.cols, s.full_off + (r0 + g * 32) * s.cols,
                                 info.cnt_off + g, expected, info.ran_index))
            else:
                for b in range(0, s.shard_numel, ITEM_ELEMS):
                    rows.append((s.shard_off + b, min(ITEM_ELEMS, s.shard_numel - b), -1, -1, 0, -1))
        for r in rows:
            assert r[0] % 4 == 0 and (r[2] < 0 or r[2] % 4 == 0), "shard_update items must be 16-byte aligned"
        return torch.tensor(rows, dtype=torch.int64).reshape(-1, 6).to(p.device)

    def view(self, name: str) -> torch.Tensor:
        start = self.region[name]
        return self.buf32[start: start + self.params.shard_numel]

    def reset_step(self) -> None:
        """Start of every step: zero the arrival counts this rank owns and the push flags, start the
        gathers (the first weight now, the others inside the GEMMs before their first use) and
        mark every F1 weight as not yet used this step.

        The inbox needs no clearing: every region that is waited on is overwritten each step.
        """
        self.counters.zero_()
        self.local_counts.zero_()
        self._push_queue.clear()
        self._gathered = set()
        for info in self.f1.values():
            info.pending = True
        if self.order is None:
            self._recording = []
            self._gather_queue = deque()
        else:
            self._gather_queue = deque(self.order)
            self._run_standalone(self._gather_queue.popleft(), None)

    def before_use(self, info: F1Info) -> None:
        """Called right before each GEMM that reads an F1 weight: at its first use of the step the
        resident copy must be gathered (by a job of an earlier GEMM, or here, standalone)."""
        if not info.pending:
            return
        info.pending = False
        if self.order is None:
            self._recording.append(info)
        if info.fqn not in self._gathered:
            try:
                self._gather_queue.remove(info)
            except ValueError:
                pass
            self._run_standalone(info, None)

    def queue_push(self, info: F2Info) -> None:
        """The weight's gradient is final for this step: the next GEMM launched pushes it."""
        self._push_queue.append(info)

    def take_jobs(self) -> Optional[torch.Tensor]:
        """Job source of every GEMM launch: at most one gather and one push."""
        g = self._gather_queue.popleft() if self._gather_queue else None
        p = self._push_queue.popleft() if self._push_queue else None
        if g is None and p is None:
            return None
        if g is not None:
            self._gathered.add(g.fqn)
        return self._descriptor(g, p)

    def flush(self) -> None:
        """End of the backward: run the pushes no GEMM took; fix the first-use order once known."""
        while self._push_queue:
            self._run_standalone(None, self._push_queue.popleft())
        if self.order is None and self._recording:
            self.order = list(self._recording)

    def _run_standalone(self, g: Optional[F1Info], p: Optional[F2Info]) -> None:
        from .._native import cuda
        if g is not None:
            self._gathered.add(g.fqn)
        cuda().copy_jobs(self._descriptor(g, p), self.params.device.index)

    def _descriptor(self, g: Optional[F1Info], p: Optional[F2Info]) -> torch.Tensor:
        """CPU int64 [16] job descriptor (layout: decode_copy_jobs in gemm_tcgen05.cu)."""
        key = (None if g is None else g.fqn, None if p is None else p.fqn)
        d = self._desc_cache.get(key)
        if d is None:
            v = [0] * 16
            if g is not None:
                v[0:5] = [g.src.data_ptr(), g.dst.data_ptr(), g.dst.shape[0], g.dst.numel() // g.dst.shape[0],
                          g.chunk_rows]
            if p is not None:
                rows, cols = p.src.shape[0], p.src.numel() // p.src.shape[0]
                v[5:15] = [p.src.data_ptr(), self.base32.data_ptr(), p.inbox_off, self.params.shard_numel, p.cnt_off,
                           rows, cols, p.chunk_rows, self.rank, self.local_counts[p.ran_index:].data_ptr()]
            d = torch.tensor(v, dtype=torch.int64)
            self._desc_cache[key] = d
        return d

    def set_f2_enabled(self, enabled: bool) -> None:
        for info in self.f2.values():
            info.enabled = enabled

    def attach(self) -> None:
        """Bind the F1/F2 metadata to the module parameters and their resident / gradient
        buffers, and register the GEMM job source."""
        from ..ops import gemm as G
        for s in self.params.slots:
            if s.fqn in self.f1:
                self.f1[s.fqn].dst = self.params.full_view(self.params.compute, s)
                s.param._f1 = self.f1[s.fqn]
            if s.fqn in self.f2:
                self.f2[s.fqn].src = self.params.full_view(self.params.grad, s)
                s.param._f2 = self.f2[s.fqn]
                s.param._f2_pending = 0
        self._desc_cache.clear()
        G.set_job_source(self.take_jobs)

    def update(self, items: Optional[torch.Tensor] = None) -> None:
        """Step-end optimizer for this rank's shards (waits for the F2 pushes it owns)."""
        from .._native import cuda
        p = self.params
        r = self.region
        offs = [r["master"], r["exp_avg"] if p.exp_avg is not None else -1, r["exp_avg_sq"],
                r["param_ema"] if p.param_ema is not None else -1, r["grad_shard"], r["inbox"], p.shard_numel]
        cuda().shard_update(self.items if items is None else items, self.buf32, offs, p.grad, self.buf16,
                            self.local_counts, self.world, self.rank, p.hyper,
                            p.beta1, p.beta2, p.weight_decay, p.ema if p.ema is not None else 0.0)


def before_use(w) -> None:
    """Make sure a sharded weight's resident copy is current before a GEMM reads it."""
    info = getattr(w, "_f1", None)
    if info is not None and info.pending:
        info.owner.before_use(info)
