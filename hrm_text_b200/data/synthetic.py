"""Synthetic PrefixLM data with the benchmark's document distribution.

Documents have log-normal packed lengths (median ``median``, clipped to ``[min_len,
max_seq_len]``), a prefix (instruction) fraction uniform in ``[0, max_prefix_frac]`` and token
ids uniform over the vocabulary. ``write_dataset`` stores them in the on-disk format that
``V1Dataset`` and the reference loader read; ``packed_batches`` runs the same multipack
sampler in memory and yields ready batches for benchmarks.
"""
from __future__ import annotations

import json
import os
from typing import Iterator

import numpy as np

from .dataset import assemble_batch
from .multipack import MultipackDistributedBatchSampler


def sample_documents(num_docs: int, vocab: int, max_seq_len: int, seed: int = 0, median: float = 512.0,
                     sigma: float = 1.0, min_len: int = 16, max_prefix_frac: float = 0.5):
    """Returns ``(inst_lens, resp_lens, tokens)``; a document packs to ``inst + resp - 1`` tokens."""
    rng = np.random.default_rng(seed)
    packed = np.clip(np.round(rng.lognormal(np.log(median), sigma, num_docs)), min_len, max_seq_len).astype(np.int64)
    prefix = np.floor(rng.uniform(0.0, max_prefix_frac, num_docs) * packed).astype(np.int64)
    inst = np.maximum(prefix, 1)
    resp = packed + 1 - inst  # >= 2 because prefix <= packed / 2 and packed >= 2
    tokens = rng.integers(0, vocab, int((inst + resp).sum()), dtype=np.int32)
    return inst, resp, tokens


def write_dataset(path: str, num_docs: int, vocab: int, max_seq_len: int, epochs: int = 1, seed: int = 0,
                  **kwargs) -> str:
    os.makedirs(path, exist_ok=True)
    inst, resp, tokens = sample_documents(num_docs, vocab, max_seq_len, seed=seed, **kwargs)
    starts = np.concatenate([[0], np.cumsum(inst + resp)[:-1]]).astype(np.int64)
    inst_start, resp_start = starts, starts + inst
    np.save(os.path.join(path, "tokens.npy"), tokens)
    meta = {"tokenizer_info": {"vocab_size": int(vocab)}, "vocab_size": None,
            "max_seq_len": int(max_seq_len) + 1, "total_length": int((inst + resp).sum())}
    with open(os.path.join(path, "metadata.json"), "w") as f:
        json.dump(meta, f)
    rng = np.random.default_rng(seed + 1)
    for e in range(epochs):
        perm = rng.permutation(num_docs)
        d = os.path.join(path, f"epoch_{e}")
        os.makedirs(d, exist_ok=True)
        for name, arr in (("inst_start", inst_start), ("inst_len", inst), ("resp_start", resp_start),
                          ("resp_len", resp)):
            np.save(os.path.join(d, f"{name}.npy"), arr[perm])
    return path


def packed_batches(tokens_per_rank: int, vocab: int, max_seq_len: int, rank: int = 0, world: int = 1,
                   seed: int = 0, num_batches: int = 4, **kwargs) -> Iterator[tuple[dict, dict]]:
    """Yield ``num_batches`` packed batches for ``rank`` (same plan on every rank)."""
    docs_needed = max(64, int(2.5 * num_batches * world * tokens_per_rank / 512)) + 16
    inst, resp, tokens = sample_documents(docs_needed, vocab, max_seq_len, seed=seed, **kwargs)
    starts = np.concatenate([[0], np.cumsum(inst + resp)[:-1]])
    sampler = MultipackDistributedBatchSampler(tokens_per_rank, inst + resp - 1, num_replicas=world, rank=rank,
                                               drop_last_batch=True)
    produced = 0
    for indices in sampler.iter():
        insts = [tokens[starts[i]: starts[i] + inst[i]] for i in indices]
        resps = [tokens[starts[i] + inst[i]: starts[i] + inst[i] + resp[i]] for i in indices]
        yield assemble_batch(insts, resps, tokens_per_rank)
        produced += 1
        if produced >= num_batches:
            return
    if produced < num_batches:
        raise RuntimeError("not enough synthetic documents for the requested number of batches")
