"""Export a training checkpoint to a Hugging Face ``hrm_text`` directory.

    python -m conversion.convert_to_hf --ckpt_path CKPT --out_dir OUT [--ckpt_epoch E]
        [--ckpt_use_ema true|false] [--tokenizer_path PATH]

Writes ``config.json`` (``model_type: hrm_text``), ``model.safetensors`` and the tokenizer.
The key mapping and the config fields are the ones the HRM-Text Hugging Face model reads
(reference conversion/convert_to_hf.py:16-97):

* ``model.{H,L}_level.core.layers.*`` -> ``model.{H,L}_module.layers.*``;
* ``model.zL_init`` -> ``model.z_L_init``; ``embed_tokens.embedding_weight`` ->
  ``model.embed_tokens.weight``; RoPE caches and ``model.zH_init`` are dropped;
* ``L_bp_steps`` lists, per H cycle, how many of its L calls train with gradients at the
  final ``bp_max_steps`` (H calls are served first, L keeps the rest).
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path
from typing import Optional

import torch

_DROP_PREFIXES = ("model.H_level.core.rotary_emb.", "model.L_level.core.rotary_emb.")
_DROP_KEYS = {"model.zH_init"}
_RENAMES = (("model.H_level.core.layers.", "model.H_module.layers."),
            ("model.L_level.core.layers.", "model.L_module.layers."),
            ("model.zL_init", "model.z_L_init"))


def remap_key(key: str) -> Optional[str]:
    if key in _DROP_KEYS or key.startswith(_DROP_PREFIXES):
        return None
    if key == "embed_tokens.embedding_weight":
        return "model.embed_tokens.weight"
    for old, new in _RENAMES:
        key = key.replace(old, new)
    return key


def convert_state_dict(state: dict[str, torch.Tensor]) -> tuple[dict[str, torch.Tensor], list[str]]:
    out, dropped = {}, []
    for k, v in state.items():
        nk = remap_key(k)
        if nk is None:
            dropped.append(k)
        else:
            out[nk] = v.detach().contiguous().cpu()
    return out, dropped


def intermediate_size(hidden: int, expansion: float) -> int:
    return ((round(expansion * hidden * 2 / 3) + 255) // 256) * 256


def l_bp_steps_per_cycle(cfg: dict) -> list[int]:
    H, L = int(cfg["H_cycles"]), int(cfg["L_cycles"])
    bp = int(cfg.get("bp_max_steps", cfg.get("max_bp_steps", H + 1)))
    h_bp = min(H, max(0, bp - 1))
    l_bp = min(H * L, max(0, bp - h_bp))
    first_grad = H * L - l_bp  # L calls with index >= first_grad train
    return [max(0, min(L, (i + 1) * L - first_grad)) for i in range(H)]


def build_hf_config(cfg: dict, tokenizer) -> dict:
    hidden = cfg["hidden_size"]
    init_type, init_std = cfg.get("init_type", "fixed_normal"), cfg.get("init_std")
    if init_type == "lecun_normal":
        in_std = 1.0 / math.sqrt(hidden)
    elif init_std is not None:
        in_std = init_std
    else:
        in_std = 1.0 / math.sqrt(hidden) if init_type == "megatron" else 0.02
    hf = {
        "model_type": "hrm_text",
        "architectures": ["HrmTextForCausalLM"],
        "vocab_size": cfg["vocab_size"],
        "hidden_size": hidden,
        "intermediate_size": intermediate_size(hidden, cfg.get("expansion", 4.0)),
        "num_hidden_layers": cfg["n_layers"],
        "num_attention_heads": cfg["num_heads"],
        "num_key_value_heads": cfg["num_heads"],
        "head_dim": hidden // cfg["num_heads"],
        "H_cycles": cfg["H_cycles"],
        "L_cycles": cfg["L_cycles"],
        "L_bp_steps": l_bp_steps_per_cycle(cfg),
        "max_position_embeddings": cfg["max_seq_len"],
        "rms_norm_eps": cfg.get("norm_eps", 1e-6),
        "rope_theta": cfg.get("rope_theta", 10000.0),
        "tie_word_embeddings": False,
        "initializer_range": in_std,
        "embedding_scale": 1.0 / in_std,
        "prefix_lm": True,
        "pad_token_id": (getattr(tokenizer, "pad_token_id", None) or 0) if tokenizer is not None else 0,
    }
    if tokenizer is not None:
        for key, name in (("bos_token_id", "boq"), ("eos_token_id", "eoa")):
            if name in cfg:
                hf[key] = tokenizer.convert_tokens_to_ids(cfg[name])
    return {k: v for k, v in hf.items() if v is not None}


def _bool(text: str) -> bool:
    return text.lower() in {"1", "true", "yes", "y"}


def convert(ckpt_path: Path, out_dir: Path, ckpt_epoch: Optional[int] = None, use_ema: bool = True,
            tokenizer_path: Optional[Path] = None, with_tokenizer: bool = True) -> dict:
    from safetensors.torch import save_file

    from hrm_text_b200.inference.engine import load_model_from_checkpoint
    from hrm_text_b200.runtime.factory import model_config_dict
    model, _carry, cfg, meta = load_model_from_checkpoint(str(ckpt_path), ckpt_epoch, use_ema,
                                                          device=torch.device("cpu"))
    full_cfg = model_config_dict(cfg.arch.model_dump(), meta.model_dump(), cfg.data.model_dump())
    tokenizer = None
    if with_tokenizer:
        from transformers import AutoTokenizer
        path = tokenizer_path or Path(meta.tokenizer_info["tokenizer_path"])
        path = path.parent if path.name == "tokenizer.json" else path
        tokenizer = AutoTokenizer.from_pretrained(str(path), use_fast=True)
        if "boq" in meta.tokenizer_info:
            tokenizer.bos_token = meta.tokenizer_info["boq"]
        if "eoa" in meta.tokenizer_info:
            tokenizer.eos_token = meta.tokenizer_info["eoa"]
    state, dropped = convert_state_dict(model.state_dict())
    print(f"[convert] mapped {len(state)} tensors; dropped {len(dropped)}")
    out_dir.mkdir(parents=True, exist_ok=True)
    hf_cfg = build_hf_config(full_cfg | meta.tokenizer_info, tokenizer)
    (out_dir / "config.json").write_text(json.dumps(hf_cfg, indent=2))
    save_file(state, str(out_dir / "model.safetensors"))
    if tokenizer is not None:
        tokenizer.save_pretrained(str(out_dir))
    print(f"[convert] wrote checkpoint to {out_dir}")
    return hf_cfg


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ckpt_path", type=Path, required=True)
    ap.add_argument("--ckpt_epoch", type=int, default=None)
    ap.add_argument("--ckpt_use_ema", type=_bool, default=True)
    ap.add_argument("--out_dir", type=Path, required=True)
    ap.add_argument("--tokenizer_path", type=Path, default=None)
    args = ap.parse_args(argv)
    convert(args.ckpt_path, args.out_dir, args.ckpt_epoch, args.ckpt_use_ema, args.tokenizer_path)


if __name__ == "__main__":
    main()
