"""scripts/prepare_sft_data.py: empty responses are dropped and the output trains (reference
scripts/test_prepare_sft_filter.py checks the same filter)."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
SPECIALS = ["<|im_start|>", "<|im_end|>", "<|box_end|>", "<|object_ref_start|>", "<|object_ref_end|>",
            "<|quad_start|>", "<|quad_end|>"]


def _tokenizer(path: Path) -> Path:
    from tokenizers import Tokenizer, models, pre_tokenizers
    words = ["[UNK]"] + SPECIALS + "what is 2+2 ? 4 capital of france paris hello hi there empty response sample a b".split()
    tok = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.add_special_tokens(SPECIALS)
    out = path / "tokenizer.json"
    tok.save(str(out))
    return out


def test_prepare_filters_empty_responses(tmp_path):
    tok = _tokenizer(tmp_path)
    rows = [{"instruction": "what is 2+2 ?", "response": "4"},
            {"instruction": "capital of france ?", "response": "paris"},
            {"instruction": "empty response sample a", "response": ""},
            {"instruction": "hello ?", "response": "hi there", "condition": "cot"},
            {"instruction": "empty response sample b", "response": ""}]
    jsonl = tmp_path / "in.jsonl"
    jsonl.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    out = tmp_path / "out"
    res = subprocess.run([sys.executable, str(ROOT / "scripts" / "prepare_sft_data.py"), "--train", str(jsonl),
                          "--tokenizer", str(tok), "--output", str(out), "--epochs", "2"],
                         capture_output=True, text=True, cwd=ROOT)
    assert res.returncode == 0, res.stderr
    assert "Skipped 2 samples with empty response" in res.stdout
    for e in range(2):
        lens = np.load(out / f"epoch_{e}" / "resp_len.npy")
        assert lens.size == 3 and (lens > 1).all()
    meta = json.loads((out / "metadata.json").read_text())
    assert meta["vocab_size"] is None and meta["max_seq_len"] == 4097

    from hrm_text_b200.data.dataset import V1Dataset, V1DatasetConfig
    ds = V1Dataset(V1DatasetConfig(seed=0, dataset_path=str(out), batch_max_length=64, drop_last_batch=False,
                                   target_only=True, rank=0, num_replicas=1))
    batch, info = next(iter(ds))
    assert info["numseqs"] >= 1 and int(batch["labels"].ne(-100).sum()) > 0
