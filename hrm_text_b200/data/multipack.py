"""Multipack distributed batch sampler (reference multipack_sampler.py:113-179).

Every rank computes the same global plan without communication and keeps bin ``rank``.
The allocator itself is native C++ (``csrc/host/multipack.cpp``); ``lpt_check_py`` /
``lpt_with_result_py`` / ``allocate_py`` below are a direct pure-Python statement of the
same algorithm, used by the tests to pin the C++ plan.
"""
from __future__ import annotations

from typing import Iterator, Optional

import numpy as np

from .._native import host


class MultipackDistributedBatchSampler:
    def __init__(self, batch_max_length: int, lengths: np.ndarray, num_replicas: Optional[int] = None,
                 rank: Optional[int] = None, drop_last_batch: bool = False):
        if num_replicas is None or rank is None:
            import torch.distributed as dist
            num_replicas = dist.get_world_size() if num_replicas is None else num_replicas
            rank = dist.get_rank() if rank is None else rank
        assert isinstance(lengths, np.ndarray)
        self.num_replicas = int(num_replicas)
        self.rank = int(rank)
        self.drop_last_batch = drop_last_batch
        self.batch_max_length = int(batch_max_length)
        self.lengths = lengths
        self.eff_total_used = 0
        self.eff_total_slots = 0

    def iter(self) -> Iterator[np.ndarray]:
        batches, used, slots = host().plan_epoch(self.lengths.astype(np.int64), self.rank,
                                                 self.batch_max_length, self.num_replicas, self.drop_last_batch)
        self.eff_total_used += used
        self.eff_total_slots += slots
        yield from batches

    __iter__ = iter

    def estimate_num_batches(self) -> int:
        return round(float(np.sum(self.lengths)) / (self.num_replicas * self.batch_max_length))

    def efficiency(self) -> float:
        return self.eff_total_used / max(1, self.eff_total_slots)


# ----------------------------------------------------------------------------------------
# pure-Python statement of the allocator (test oracle)
# ----------------------------------------------------------------------------------------

def _sift(load: list, ids: Optional[list], n: int) -> None:
    u = 1
    while 2 * u <= n:
        v = 2 * u
        if v + 1 <= n and load[v + 1] < load[v]:
            v += 1
        if load[u] <= load[v]:
            break
        load[u], load[v] = load[v], load[u]
        if ids is not None:
            ids[u], ids[v] = ids[v], ids[u]
        u = v


def lpt_check_py(lengths, c: int, n: int) -> bool:
    load = [0] * (n + 1)
    for x in sorted((int(v) for v in lengths), reverse=True):
        load[1] += x
        if load[1] > c:
            return False
        _sift(load, None, n)
    return True


def lpt_with_result_py(lengths, n: int, rank: int) -> np.ndarray:
    lengths = [int(v) for v in lengths]
    order = sorted(range(len(lengths)), key=lambda i: lengths[i])[::-1]  # stable ascending, reversed
    load = [0] * (n + 1)
    ids = list(range(-1, n))
    mine = []
    for i in order:
        load[1] += lengths[i]
        if ids[1] == rank:
            mine.append(i)
        _sift(load, ids, n)
    return np.array(mine, dtype=np.int64)


def allocate_py(lengths: np.ndarray, start: int, rank: int, c: int, n: int):
    total, end = 0, start
    while end < lengths.size:
        total += int(lengths[end])
        end += 1
        if total >= c * n:
            break
    run = lengths[start:end]
    lo, hi = 1, 1 + run.size
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if lpt_check_py(run[:mid], c, n):
            lo = mid
        else:
            hi = mid
    return lo >= n, lo, start + lpt_with_result_py(run[:lo], n, rank), int(np.sum(run[:lo]))
