"""Sharded engine over gloo: 2 ranks must follow the 1-rank trajectory.

Tiny HRM-Text (hidden 256, 4 heads of dim 64, SwiGLU 688, 2-layer H and L stacks, 2 H x 2 L
cycles, vocab 32768), fp32, 10 AdamATan2 steps at lr 2.5e-4, seed 0. Each rank holds one packed
sequence of 2048 tokens of documents with lengths uniform in [64, 1024] (the last truncated)
and prefixes uniform in [0, len/2]; only response tokens carry labels. The single-rank run
trains on both sequences concatenated. The loss divisor is the global mean token count and
the SUM-reduced gradient is then 2x the single-rank one, which AdamATan2 ignores
(atan2 is scale invariant), so the parameters must match.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hrm_text_b200.runtime.engine import TrainEngine
from hrm_text_b200.runtime.factory import arch_preset, build_model

STEPS, SEQ, VOCAB = 10, 2048, 32768


def cfg():
    return arch_preset("hrm", "L") | dict(n_layers=4, hidden_size=256, num_heads=4, intermediate_size_override=688,
                                          H_cycles=2, L_cycles=2, vocab_size=VOCAB, max_seq_len=1024)


def packed_sequence(seed: int):
    rng = np.random.default_rng(seed)
    lens, total = [], 0
    while total < SEQ:
        L = min(int(rng.integers(64, 1025)), SEQ - total)
        lens.append(L)
        total += L
    inputs = rng.integers(0, VOCAB, SEQ).astype(np.int32)
    labels = rng.integers(0, VOCAB, SEQ).astype(np.int32)
    pos = np.zeros(SEQ, np.int32)
    prefixes = []
    start = 0
    for L in lens:
        p = int(rng.integers(0, L // 2 + 1))
        prefixes.append(p)
        labels[start:start + p] = -100
        pos[start:start + L] = np.arange(L)
        start += L
    return inputs, labels, pos, np.array(lens), np.array(prefixes)


def batch_from(parts):
    inputs = np.concatenate([p[0] for p in parts])
    labels = np.concatenate([p[1] for p in parts])
    pos = np.concatenate([p[2] for p in parts])
    lens = np.concatenate([p[3] for p in parts])
    prefixes = np.concatenate([p[4] for p in parts])
    T = inputs.size
    cu = np.zeros(T, np.int32)
    cu[1:lens.size + 1] = np.cumsum(lens)
    pl = np.zeros(T, np.int32)
    pl[:lens.size] = prefixes
    causal = np.zeros(T, np.int32)
    causal[:lens.size] = lens - prefixes
    t = torch.from_numpy
    return dict(inputs=t(inputs), labels=t(labels), position_ids=t(pos), prefix_lens=t(pl), causal_lens=t(causal),
                cu_seqlens=t(cu))


def train(batches_per_step, world=1, rank=0):
    torch.manual_seed(0)
    eng = TrainEngine(build_model(cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=None)
    losses = []
    for batch in batches_per_step:
        loss, _ = eng.train_step(batch, lr=2.5e-4, bp_steps=5)
        losses.append(float(loss))
    full = {s.fqn: eng.params.full_param_fp32(s) for s in eng.params.slots}
    return full, losses


def _rank_main(rank, world, out, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))
    try:
        batches = [batch_from([packed_sequence(1000 * s + rank)]) for s in range(STEPS)]
        full, losses = train(batches, world, rank)
        if rank == 0:
            torch.save((full, losses), out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_match_one_rank(tmp_path, world):
    """world 4 also exercises dim-0 chunks with padding (rows not divisible by the world)."""
    out = str(tmp_path / f"w{world}.pt")
    mp.spawn(_rank_main, args=(world, out, 29681 + world), nprocs=world, join=True)
    full2, losses2 = torch.load(out)
    batches = [batch_from([packed_sequence(1000 * s + r) for r in range(world)]) for s in range(STEPS)]
    full1, losses1 = train(batches)
    assert all(np.isfinite(losses1)) and all(np.isfinite(losses2))
    # Elementwise agreement to fp32 summation noise; a few elements whose gradient nearly
    # cancels can differ by one AdamATan2 step (atan2 is discontinuous at 0; one step moves a
    # weight by at most lr * (pi / 2) / (1 - beta1) ~ 4e-3).
    for k, v in full1.items():
        d = (full2[k] - v).abs()
        assert float(d.max()) < 4e-3, k
        assert int((d > 2e-5).sum()) <= max(2, v.numel() // 100000), (k, int((d > 2e-5).sum()))
