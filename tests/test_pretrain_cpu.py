"""End-to-end driver on CPU: pretrain a tiny HRM for a few steps, checkpoint, resume (SFT style)."""
import os

import torch

from hrm_text_b200.config import PretrainConfig, compose
from hrm_text_b200.data.synthetic import write_dataset
from hrm_text_b200.runtime.pretrain import lr_at, run

TINY = ["arch.n_layers=2", "arch.hidden_size=256", "arch.num_heads=2", "global_batch_size=512", "epochs=1",
        "lr_warmup_steps=2", "+log_interval=1"]


def test_lr_schedule():
    cfg = PretrainConfig(**compose("cfg_sft", ["resume_from=/x", "data.path=/y", "lr=1.0", "lr_warmup_steps=10"]))
    assert lr_at(cfg, 5, 110) == 0.5
    assert abs(lr_at(cfg, 10, 110) - 1.0) < 1e-9
    assert abs(lr_at(cfg, 110, 110) - 0.1) < 1e-9  # cosine down to lr_min_ratio
    pre = PretrainConfig(**compose("cfg_pretrain", ["lr=1.0"]))
    assert lr_at(pre, 5000, 10000) == 1.0  # constant after warm-up (lr_min_ratio 1.0)


def test_pretrain_then_resume(tmp_path, monkeypatch):
    monkeypatch.setenv("WANDB_MODE", "disabled")
    data = write_dataset(str(tmp_path / "data"), num_docs=120, vocab=500, max_seq_len=256, epochs=2, median=64.0)
    out = str(tmp_path / "ckpt")
    last = run("cfg_pretrain", TINY + [f"data.path={data}", f"+checkpoint_path={out}"], max_steps=4, num_workers=0)
    assert "train/loss" in last and torch.isfinite(torch.tensor(last["train/loss"]))
    assert os.path.isdir(os.path.join(out, "fsdp2_epoch_1"))
    assert os.path.exists(os.path.join(out, "all_config.yaml"))
    assert os.path.exists(os.path.join(out, "train_metadata.yaml"))
    sft_out = str(tmp_path / "sft")
    last2 = run("cfg_sft", TINY + [f"data.path={data}", f"resume_from={out}", f"+checkpoint_path={sft_out}",
                                   "weights_only_resume_from_ema=true"], max_steps=2, num_workers=0)
    assert "train/loss" in last2
    assert os.path.isdir(os.path.join(sft_out, "fsdp2_epoch_1"))
