"""PrefixLM packed dataset in the reference's on-disk format (reference dataset_new.py).

On disk (written by ``scripts/prepare_sft_data.py``, the ``data_io`` pipeline, or
``hrm_text_b200.data.synthetic``):

* ``metadata.json``: ``{"tokenizer_info": {..., "vocab_size": V}, "vocab_size": null,
  "max_seq_len": S, "total_length": N}``;
* ``tokens.npy``: all token ids;
* ``epoch_{e}/{inst_start,inst_len,resp_start,resp_len}.npy``: one pre-shuffled document
  order per epoch.

Each document becomes ``inputs = inst + resp[:-1]`` with labels ``-100`` over the
instruction except its last position (``target_only``), then ``resp``; positions restart
at 0 per document. A batch is the documents the multipack sampler assigns to this rank,
concatenated and padded to ``batch_max_length`` (inputs 0, labels -100, positions 0), plus
fixed-length ``prefix_lens`` / ``causal_lens`` / ``cu_seqlens`` and host scalars
(dataset_new.py:88-134, flash_attention_prefixlm_v2.py:10-24).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, fields
from typing import Any, Optional

import numpy as np
import pydantic
import torch
from torch.utils.data import IterableDataset, get_worker_info

from ..models.common import IGNORE_LABEL_ID
from ..models.layers import find_multiple
from .multipack import MultipackDistributedBatchSampler


class V1DatasetConfig(pydantic.BaseModel):
    seed: int
    dataset_path: str
    batch_max_length: int
    drop_last_batch: bool
    target_only: bool
    rank: int
    num_replicas: int


class V1DatasetMeta(pydantic.BaseModel):
    tokenizer_info: dict[str, Any] = {}
    vocab_size: Optional[int] = None
    max_seq_len: int
    total_length: int


@dataclass
class V1DatasetIndices:
    inst_start: np.ndarray
    inst_len: np.ndarray
    resp_start: np.ndarray
    resp_len: np.ndarray


def compute_aux_seq_tensors_scalars(prefix_lens: np.ndarray, causal_lens: np.ndarray, batch_max_tokens: int):
    """Fixed-length per-document arrays (padded to ``batch_max_tokens``) and host scalars."""
    total = prefix_lens + causal_lens
    n = total.shape[0]
    cu = np.zeros(batch_max_tokens, dtype=np.int32)
    cu[1:n + 1] = np.cumsum(total, dtype=np.int32)
    tensors = {
        "prefix_lens": np.pad(prefix_lens.astype(np.int32), (0, batch_max_tokens - n)),
        "causal_lens": np.pad(causal_lens.astype(np.int32), (0, batch_max_tokens - n)),
        "cu_seqlens": cu,
    }
    scalars = {"total_seqlen": int(total.sum()), "numseqs": int(n),
               "max_seqlen_prefix": int(prefix_lens.max()), "max_seqlen_causal": int(causal_lens.max()),
               "max_seqlen_all": int(total.max())}
    return tensors, scalars


def assemble_batch(insts: list[np.ndarray], resps: list[np.ndarray], batch_max_length: int, target_only: bool = True):
    """Pack documents (instruction, response token arrays) into one fixed-length batch."""
    inputs, labels, positions = [], [], []
    prefix, causal = [], []
    for inst, resp in zip(insts, resps):
        inst = inst.astype(np.int32)
        resp = resp.astype(np.int32)
        inputs += [inst, resp[:-1]]
        labels += [np.full(len(inst) - 1, IGNORE_LABEL_ID, dtype=np.int32) if target_only else inst[1:], resp]
        positions.append(np.arange(len(inst) + len(resp) - 1, dtype=np.int32))
        prefix.append(len(inst))
        causal.append(len(resp) - 1)
    batch = {"inputs": np.concatenate(inputs), "labels": np.concatenate(labels),
             "position_ids": np.concatenate(positions)}
    pad = batch_max_length - batch["inputs"].shape[0]
    assert pad >= 0, f"packed batch ({batch['inputs'].shape[0]} tokens) exceeds batch_max_length {batch_max_length}"
    fill = {"inputs": 0, "labels": IGNORE_LABEL_ID, "position_ids": 0}
    for key, value in fill.items():
        batch[key] = np.pad(batch[key], (0, pad), constant_values=value)
    tensors, scalars = compute_aux_seq_tensors_scalars(np.array(prefix, dtype=np.int32),
                                                       np.array(causal, dtype=np.int32), batch_max_length)
    return {k: torch.from_numpy(v) for k, v in (batch | tensors).items()}, scalars


class V1Dataset(IterableDataset):
    def __init__(self, config: V1DatasetConfig):
        super().__init__()
        self.config = config
        self.metadata = self._load_metadata()
        self._data: Optional[np.ndarray] = None
        self._indices: Optional[V1DatasetIndices] = None
        self._sampler: Optional[MultipackDistributedBatchSampler] = None
        self._epoch = 0

    def _load_metadata(self) -> V1DatasetMeta:
        with open(os.path.join(self.config.dataset_path, "metadata.json")) as f:
            meta = V1DatasetMeta(**json.load(f))
        meta.max_seq_len -= 1  # autoregressive shift
        assert meta.vocab_size is None, "metadata.json must leave vocab_size null (it is derived)"
        meta.vocab_size = find_multiple(meta.tokenizer_info.pop("vocab_size"), 256)
        return meta

    def _begin_epoch(self) -> None:
        root = self.config.dataset_path
        if self._data is None:
            self._data = np.load(os.path.join(root, "tokens.npy"), mmap_mode="r")
        self._indices = V1DatasetIndices(**{
            f.name: np.load(os.path.join(root, f"epoch_{self._epoch}", f"{f.name}.npy"), mmap_mode="r")
            for f in fields(V1DatasetIndices)})
        self._epoch += 1
        self._sampler = MultipackDistributedBatchSampler(
            lengths=np.asarray(self._indices.inst_len + self._indices.resp_len - 1),
            batch_max_length=self.config.batch_max_length, drop_last_batch=self.config.drop_last_batch,
            rank=self.config.rank, num_replicas=self.config.num_replicas)

    def _load_batch(self, indices: np.ndarray):
        assert self._data is not None and self._indices is not None
        idx = self._indices
        insts = [self._data[s: s + l] for s, l in zip(idx.inst_start[indices], idx.inst_len[indices])]
        resps = [self._data[s: s + l] for s, l in zip(idx.resp_start[indices], idx.resp_len[indices])]
        return assemble_batch(insts, resps, self.config.batch_max_length, self.config.target_only)

    def __iter__(self):
        info = get_worker_info()
        assert info is None or info.num_workers == 1
        self._begin_epoch()
        assert self._sampler is not None
        for indices in self._sampler.iter():
            yield self._load_batch(indices)
