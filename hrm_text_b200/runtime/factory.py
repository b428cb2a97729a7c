"""Model construction from configuration (reference pretrain.py:131-164)."""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from ..registry import load_model_class


def model_config_dict(arch: dict, metadata: dict, data: Optional[dict] = None) -> dict:
    """``arch | train_metadata | data`` as the reference merges them (pretrain.py:132)."""
    return dict(arch) | dict(metadata) | dict(data or {})


def build_model(config_dict: dict, device: torch.device | str = "cpu") -> nn.Module:
    """Instantiate ``arch.name`` wrapped by ``arch.head`` with parameters on ``device`` (fp32)."""
    model_cls = load_model_class(config_dict["name"])
    head_cls = load_model_class(config_dict["head"])
    with torch.device(device):
        model = model_cls(config_dict)
        return head_cls(model, config_dict)


def arch_preset(net: str = "hrm", size: str = "L", **overrides) -> dict:
    """Compose ``arch/net/<net>.yaml`` and ``arch/size/<size>.yaml`` into one arch dict."""
    from ..config import compose
    tree = compose("cfg_pretrain", [f"arch/net@arch={net}", f"arch/size@arch={size}", "data.path=unused"])
    return tree["arch"] | overrides
