import pytest

from hrm_text_b200.config import PretrainConfig, compose, parse_cli


def test_default_pretrain_config():
    tree = compose("cfg_pretrain")
    cfg = PretrainConfig(**tree)
    assert cfg.arch.name == "baselines.hrm_nocarry_bp_warmup@HierarchicalReasoningModel"
    assert cfg.arch.model_extra["hidden_size"] == 1536 and cfg.arch.model_extra["n_layers"] == 32
    assert cfg.global_batch_size == 196608 and cfg.lr == 2.2e-4 and cfg.ema == 0.9999
    assert cfg.data.path == "/dev/shm/sampled"


def test_size_and_value_overrides():
    tree = compose("cfg_pretrain", ["arch/size@arch=L", "lr=2.5e-4", "global_batch_size=172032", "+checkpoint_path=/x",
                                    "arch.bp_max_steps=4"])
    cfg = PretrainConfig(**tree)
    assert cfg.arch.model_extra["hidden_size"] == 1280 and cfg.lr == 2.5e-4
    assert cfg.global_batch_size == 172032 and cfg.checkpoint_path == "/x"
    assert cfg.arch.model_extra["bp_max_steps"] == 4


def test_unknown_key_needs_plus():
    with pytest.raises(KeyError):
        compose("cfg_pretrain", ["nonexistent_key=1"])


def test_sft_mandatory_values():
    with pytest.raises(ValueError):
        compose("cfg_sft", [])
    tree = compose("cfg_sft", ["resume_from=/ckpt", "data.path=/data", "arch/size@arch=L"])
    cfg = PretrainConfig(**tree)
    assert cfg.arch.model_extra["bp_warmup_ratio"] == 0.0 and cfg.lr_min_ratio == 0.1


def test_parse_cli():
    name, ov = parse_cli(["--config-name", "cfg_sft", "lr=1"])
    assert name == "cfg_sft" and ov == ["lr=1"]
    name, ov = parse_cli(["--config-name=cfg_sft"])
    assert name == "cfg_sft" and ov == []


@pytest.mark.parametrize("net", ["hrm", "rins", "transformer", "trm", "trm_match_recurrence", "ut"])
def test_every_net_composes(net):
    tree = compose("cfg_pretrain", [f"arch/net@arch={net}"])
    assert "@" in tree["arch"]["name"]
