import numpy as np
import torch

from hrm_text_b200.data.dataset import V1Dataset, V1DatasetConfig, assemble_batch
from hrm_text_b200.data.synthetic import write_dataset
from hrm_text_b200.models.common import IGNORE_LABEL_ID


def test_assemble_batch_semantics():
    inst = [np.array([5, 6, 7]), np.array([9])]
    resp = [np.array([1, 2]), np.array([3, 4, 8])]
    b, s = assemble_batch(inst, resp, 12)
    assert b["inputs"].tolist() == [5, 6, 7, 1, 9, 3, 4, 0, 0, 0, 0, 0]
    assert b["labels"].tolist() == [-100, -100, 1, 2, 3, 4, 8, -100, -100, -100, -100, -100]
    assert b["position_ids"].tolist() == [0, 1, 2, 3, 0, 1, 2, 0, 0, 0, 0, 0]
    assert b["prefix_lens"][:3].tolist() == [3, 1, 0]
    assert b["causal_lens"][:3].tolist() == [1, 2, 0]
    assert b["cu_seqlens"][:4].tolist() == [0, 4, 7, 0]
    assert s == {"total_seqlen": 7, "numseqs": 2, "max_seqlen_prefix": 3, "max_seqlen_causal": 2, "max_seqlen_all": 4}
    b2, _ = assemble_batch(inst, resp, 12, target_only=False)
    assert b2["labels"][:4].tolist() == [6, 7, 1, 2]


def test_dataset_roundtrip(tmp_path):
    path = write_dataset(str(tmp_path / "d"), num_docs=300, vocab=1000, max_seq_len=256, epochs=2, median=64)
    cfg = V1DatasetConfig(seed=0, dataset_path=path, batch_max_length=1024, drop_last_batch=True, target_only=True,
                          rank=0, num_replicas=2)
    ds = V1Dataset(cfg)
    assert ds.metadata.vocab_size == 1024 and ds.metadata.max_seq_len == 256
    batches = list(iter(ds))
    assert len(batches) > 3
    for b, s in batches:
        assert b["inputs"].shape == (1024,)
        total = s["total_seqlen"]
        cu = b["cu_seqlens"][: s["numseqs"] + 1]
        assert cu[-1].item() == total
        assert (b["labels"][total:] == IGNORE_LABEL_ID).all()
        assert int(b["inputs"].max()) < 1000
    assert len(list(iter(ds))) > 3  # second epoch
