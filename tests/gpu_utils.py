"""Helpers shared by the GPU tests: random packed batches and tolerance checks."""
import numpy as np
import torch


def random_packing(T: int, seed: int = 0, max_doc: int = 700, causal_frac: bool = True, pad: int = 37):
    """Documents with varied lengths (including 1 and prefix 0 / prefix == len), padded tail."""
    rng = np.random.default_rng(seed)
    lens, total = [], 0
    special = [1, 2, 130, 129, 64]
    while True:
        L = special.pop(0) if special else int(rng.integers(1, max_doc))
        if total + L > T - pad:
            break
        lens.append(L)
        total += L
    prefixes = []
    for i, L in enumerate(lens):
        if i % 5 == 0:
            prefixes.append(0)
        elif i % 5 == 1:
            prefixes.append(L)
        else:
            prefixes.append(int(rng.integers(0, L // 2 + 1)))
    cu = np.zeros(T, dtype=np.int32)
    cu[1:len(lens) + 1] = np.cumsum(lens)
    pl = np.zeros(T, dtype=np.int32)
    pl[:len(lens)] = prefixes
    pos = np.zeros(T, dtype=np.int32)
    for s, L in zip(cu[:len(lens)], lens):
        pos[s:s + L] = np.arange(L)
    return torch.from_numpy(cu), torch.from_numpy(pl), torch.from_numpy(pos), total


def assert_close(actual, expected, rel=2e-2, name=""):
    actual = actual.float()
    expected = expected.float()
    scale = expected.abs().max().item() + 1e-6
    err = (actual - expected).abs().max().item()
    assert err <= rel * scale, f"{name}: max abs err {err:.4g} vs scale {scale:.4g} (rel {err / scale:.3g})"
