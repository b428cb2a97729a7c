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


def assert_close(actual, expected, rel=2e-2, name="", atol=None):
    """Element-wise ``|actual - expected| <= atol + rel * |expected|``.

    ``atol`` defaults to ``rel`` times the RMS of ``expected`` (not its maximum), so a wrong
    region of small values -- a masked tile, a padding head, a short document -- cannot hide
    behind the largest entries of the tensor. Non-finite values always fail.
    """
    actual = actual.float()
    expected = expected.float()
    assert actual.shape == expected.shape, f"{name}: shape {tuple(actual.shape)} vs {tuple(expected.shape)}"
    assert torch.isfinite(actual).all().item(), f"{name}: non-finite values"
    if atol is None:
        atol = rel * (expected.pow(2).mean().sqrt().item() + 1e-6)
    diff = (actual - expected).abs()
    excess = diff - (atol + rel * expected.abs())
    worst = int(excess.flatten().argmax().item())
    if excess.flatten()[worst].item() > 0:
        idx = np.unravel_index(worst, tuple(actual.shape))
        raise AssertionError(
            f"{name}: element {tuple(int(i) for i in idx)} = {actual.flatten()[worst].item():.5g}, expected "
            f"{expected.flatten()[worst].item():.5g} (|diff| {diff.flatten()[worst].item():.4g} > atol {atol:.4g} "
            f"+ {rel:g}*|expected|); {(excess > 0).sum().item()} of {excess.numel()} elements out of tolerance")
