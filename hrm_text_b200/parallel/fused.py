"""Peer-memory setup for the fused collective GEMMs (multi-GPU, CUDA).

The sharding engine keeps, per rank, the fp32 master weights, AdamATan2 state and the fp32
gradient shard in one symmetric buffer, and the bf16 weight shards in another, allocated
with ``torch.distributed._symmetric_memory`` so that every rank can address every other
rank's copy directly over NVLink (peer pointers). On top of that:

* **F1 — all-gather fused with the first consuming GEMM.** The QKV and gate/up projections
  read their weight rows straight from the owning rank's bf16 shard (a per-rank TMA tensor
  map over that shard, no multicast); the CTAs of the first M row write each tile through to
  the local resident copy and publish a per-N-tile flag, so every byte crosses NVLink once
  per step and all later calls (the other recurrent cycles, the backward) read locally.
* **F2 — weight gradient fused with the reduce-scatter and the optimizer.** The last
  backward contribution to each block weight runs a wgrad GEMM whose epilogue stores each
  complete fp32 tile (plain 16-byte stores, no remote atomics) into this rank's slot of the
  owner's inbox and counts itself on the owner; the CTA that completes a tile's count sums
  the slots and applies AdamATan2 to that tile of the owner's master weights / state and
  writes the bf16 shard.

The embedding and LM head stay on NCCL (reduce-scatter + AdamATan2 kernel + all-gather).
Cross-rank ordering is provided by the collectives every step already has: the loss
divisor all-reduce separates each rank's zeroing of its gradient shard and counters from
peers' F2 reductions, and the end-of-step all-gather separates F2 updates from the next
step's F1 reads.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

F1_SUFFIXES = ("attn.gqkv_proj.weight", "mlp.gate_up_proj.weight")
F2_SUFFIXES = ("attn.gqkv_proj.weight", "attn.o_proj.weight", "mlp.gate_up_proj.weight", "mlp.down_proj.weight")
MAX_F1_TILES = 256


@dataclass
class F1Info:
    maps: torch.Tensor          # device uint8 [world * 128]: one CUtensorMap per rank's shard
    shard_rows: int
    flags: torch.Tensor         # int32 [MAX_F1_TILES], zeroed every step


@dataclass
class F2Info:
    offsets: list[int]          # grad, master, exp_avg, exp_avg_sq, ema (fp32), shard16 (bf16), counters (int32)
    shard_rows: int
    tiles: int
    owner: "FusedCollectives" = field(repr=False, default=None)
    enabled: bool = True


def choose_split(tiles: int, sms: int, max_split: int = 8) -> int:
    """Split-K factor giving the best whole-wave utilisation for ``tiles`` output tiles."""
    best, best_eff = 1, 0.0
    for s in range(1, max_split + 1):
        units = tiles * s
        eff = units / (-(-units // sms) * sms)
        if eff > best_eff + 1e-9:
            best, best_eff = s, eff
    return best


class FusedCollectives:
    """Symmetric buffers + per-weight F1/F2 metadata for one ``ShardedParameters``."""

    def __init__(self, params, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        from .._native import cuda
        self.params = params
        self.group = group or dist.group.WORLD
        self.world, self.rank = params.world, params.rank
        dev = params.device
        S = params.shard_numel
        names = ["master", "exp_avg", "exp_avg_sq", "param_ema", "grad_shard"]
        self.region = {n: i * S for i, n in enumerate(names)}
        # F2 inbox: one fp32 slot of the whole shard per source rank, [world][S]
        self.region["inbox"] = len(names) * S

        import os
        enable_f2 = os.environ.get("HRM_F2", "1") != "0"  # HRM_F2=0: block-weight gradients over NCCL
        f2_slots = [s for s in params.slots if enable_f2 and s.fqn.endswith(F2_SUFFIXES) and s.chunk_rows % 128 == 0]
        f1_slots = [s for s in params.slots if s.fqn.endswith(F1_SUFFIXES) and s.chunk_rows % 128 == 0]
        tiles = {s.fqn: (-(-s.rows // 128)) * (-(-s.cols // 256)) for s in f2_slots}
        cnt_total = sum(tiles.values())
        self.cnt_off = (len(names) + self.world) * S
        n32 = self.cnt_off + ((cnt_total + 63) // 64) * 64

        self.buf32 = symm_mem.empty(n32, dtype=torch.float32, device=dev)
        self.handle32 = symm_mem.rendezvous(self.buf32, self.group)
        self.buf16 = symm_mem.empty(S, dtype=torch.bfloat16, device=dev)
        self.handle16 = symm_mem.rendezvous(self.buf16, self.group)
        self.buf32.zero_()
        self.buf16.zero_()
        self.base32 = torch.tensor(list(self.handle32.buffer_ptrs), dtype=torch.int64, device=dev)
        self.base16 = torch.tensor(list(self.handle16.buffer_ptrs), dtype=torch.int64, device=dev)
        self.counters = self.buf32[self.cnt_off:].view(torch.int32)

        self.f1_flags = torch.zeros(max(1, len(f1_slots)) * MAX_F1_TILES, dtype=torch.int32, device=dev)
        self.f1: dict[str, F1Info] = {}
        for i, s in enumerate(f1_slots):
            addrs = [int(b) + s.shard_off * 2 for b in self.handle16.buffer_ptrs]
            maps = cuda().encode_shard_maps(addrs, s.chunk_rows, s.cols).to(dev)
            self.f1[s.fqn] = F1Info(maps, s.chunk_rows, self.f1_flags[i * MAX_F1_TILES:(i + 1) * MAX_F1_TILES])

        self.f2: dict[str, F2Info] = {}
        cnt = 0
        for s in f2_slots:
            offs = [self.region["inbox"] + s.shard_off, self.region["master"] + s.shard_off,
                    self.region["exp_avg"] + s.shard_off, self.region["exp_avg_sq"] + s.shard_off,
                    self.region["param_ema"] + s.shard_off, s.shard_off, self.cnt_off + cnt]
            self.f2[s.fqn] = F2Info(offs, s.chunk_rows, tiles[s.fqn], owner=self)
            cnt += tiles[s.fqn]

    def view(self, name: str) -> torch.Tensor:
        start = self.region[name]
        return self.buf32[start: start + self.params.shard_numel]

    def reset_step(self) -> None:
        """Zero this rank's gradient shard, F2 counters and F1 flags (start of every step).

        The inbox needs no clearing: every slot of every tile is overwritten each step.
        """
        self.view("grad_shard").zero_()
        self.counters.zero_()
        self.f1_flags.zero_()

    def set_f2_enabled(self, enabled: bool) -> None:
        for info in self.f2.values():
            info.enabled = enabled

    def attach(self) -> None:
        """Expose the F1/F2 metadata on the module parameters (read by the fused block)."""
        for s in self.params.slots:
            if s.fqn in self.f1:
                s.param._f1 = self.f1[s.fqn]
            if s.fqn in self.f2:
                s.param._f2 = self.f2[s.fqn]
                s.param._f2_pending = 0

    def f2_kernel_args(self) -> tuple:
        p = self.params
        return (self.base32, self.base16, p.hyper, p.beta1, p.beta2, p.weight_decay,
                p.ema if p.ema is not None else 0.0, p.exp_avg is not None, p.param_ema is not None)
