"""HF export: remapped keys, derived config fields, EMA weights."""
import json

import torch

from conversion.convert_to_hf import convert, l_bp_steps_per_cycle, remap_key
from hrm_text_b200.config import PretrainConfig, compose
from hrm_text_b200.data.synthetic import packed_batches
from hrm_text_b200.runtime.checkpoint import save_checkpoint, write_run_files
from hrm_text_b200.runtime.engine import TrainEngine
from hrm_text_b200.runtime.factory import build_model, model_config_dict


def test_key_remap_and_bp_steps():
    assert remap_key("model.H_level.core.layers.3.attn.o_proj.weight") == "model.H_module.layers.3.attn.o_proj.weight"
    assert remap_key("model.zL_init") == "model.z_L_init"
    assert remap_key("embed_tokens.embedding_weight") == "model.embed_tokens.weight"
    assert remap_key("model.L_level.core.rotary_emb.cos_cached") is None
    assert remap_key("lm_head.weight") == "lm_head.weight"
    assert l_bp_steps_per_cycle({"H_cycles": 2, "L_cycles": 3, "bp_max_steps": 5}) == [0, 3]
    assert l_bp_steps_per_cycle({"H_cycles": 2, "L_cycles": 3, "bp_max_steps": 6}) == [1, 3]


def test_convert_tiny_checkpoint(tmp_path):
    from safetensors.torch import load_file
    cfg = PretrainConfig(**compose("cfg_pretrain", ["arch/size@arch=L", "arch.n_layers=2", "arch.hidden_size=256",
                                                     "arch.num_heads=2", "data.path=/unused", "ema=0.5"]))
    meta = {"tokenizer_info": {}, "vocab_size": 512, "max_seq_len": 128, "total_length": 1000}
    model_cfg = model_config_dict(cfg.arch.model_dump(), meta, cfg.data.model_dump())
    torch.manual_seed(0)
    eng = TrainEngine(build_model(model_cfg), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.5)
    for b, _ in packed_batches(256, 512, 128, num_batches=2, median=32.0):
        eng.train_step(b, lr=1e-3, bp_steps=3)
    ckpt = tmp_path / "ckpt"
    write_run_files(str(ckpt), cfg.model_dump(), meta)
    save_checkpoint(eng.params, eng.model, str(ckpt), epoch=1)
    out = tmp_path / "hf"
    convert(ckpt, out, use_ema=True, with_tokenizer=False)
    hf = json.loads((out / "config.json").read_text())
    assert hf["model_type"] == "hrm_text" and hf["hidden_size"] == 256 and hf["L_bp_steps"] == [0, 3]
    assert hf["intermediate_size"] == 768 and hf["num_hidden_layers"] == 2
    tensors = load_file(str(out / "model.safetensors"))
    assert "model.H_module.layers.0.attn.gqkv_proj.weight" in tensors and "model.z_L_init" in tensors
    ema = {s.fqn: eng.params.full_param_fp32(s, eng.params.param_ema) for s in eng.params.slots}
    assert tensors["lm_head.weight"].dtype == torch.bfloat16  # forward dtype, as exported by the reference
    torch.testing.assert_close(tensors["lm_head.weight"], ema["lm_head.weight"].bfloat16())
    torch.testing.assert_close(tensors["model.embed_tokens.weight"], ema["embed_tokens.embedding_weight"].bfloat16())
