"""Transformer backbone: config, block and stack (reference models/transformer.py).

* ``TransformerConfig`` keeps the reference's fields and derived properties:
  ``intermediate_size = find_multiple(round(expansion * h * 2/3), 256)`` (transformer.py:42-46)
  and the three init schemes (transformer.py:48-62).
* ``TransformerBlock`` is a pre-norm or post-norm layer with parameter-free RMSNorm
  (transformer.py:65-96). ``Transformer`` owns the RoPE tables, the layers and, for pre-norm,
  a final RMSNorm (transformer.py:99-128).

Device split: on CPU the stack runs the plain torch modules (the oracle). On CUDA, without a
KV cache, it runs ``hrm_text_b200.ops.block.stack_forward``: every layer is one fused
autograd node built from this framework's sm_100a kernels (GEMMs with RoPE / SwiGLU /
residual epilogues, PrefixLM flash attention with the sigmoid gate fused, fused
add+RMSNorm). The CUDA path fails loudly when the extension is missing.
"""
from __future__ import annotations

import math
from typing import Literal, Optional

import torch
import torch.nn.functional as F
from pydantic import BaseModel
from torch import Tensor, nn

from .common import fused_path
from .layers import Attention, Cache, RotaryEmbedding, SwiGLU, find_multiple

AttnType = Literal["causal", "prefixlm"]


class InitConfig(BaseModel):
    in_std: float
    attn_out_std: float
    ff_out_std: float


class TransformerConfig(BaseModel):
    max_seq_len: int

    n_layers: int
    hidden_size: int
    num_heads: int
    expansion: float

    attn_type: AttnType = "prefixlm"

    init_type: Literal["fixed_normal", "lecun_normal", "megatron"]
    init_std: Optional[float] = None

    norm_type: Literal["pre", "post"]
    norm_eps: float

    pos_emb_type: Literal["rope", "none"]
    rope_theta: Optional[float] = None

    # Optional explicit SwiGLU width (not in the reference; used by small test models).
    intermediate_size_override: Optional[int] = None

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def intermediate_size(self) -> int:
        if self.intermediate_size_override is not None:
            return self.intermediate_size_override
        # GLU width matched to a vanilla MLP of the same expansion, rounded to 256.
        return find_multiple(round(self.expansion * self.hidden_size * 2 / 3), 256)

    @property
    def init_config(self) -> InitConfig:
        if self.init_type == "fixed_normal":
            std = self.init_std if self.init_std is not None else 0.02
            return InitConfig(in_std=std, attn_out_std=std, ff_out_std=std)
        if self.init_type == "lecun_normal":
            return InitConfig(in_std=1.0 / math.sqrt(self.hidden_size),
                              attn_out_std=1.0 / math.sqrt(self.hidden_size),
                              ff_out_std=1.0 / math.sqrt(self.intermediate_size))
        if self.init_type == "megatron":
            in_std = self.init_std if self.init_std is not None else 1.0 / math.sqrt(self.hidden_size)
            out_std = in_std / math.sqrt(2.0 * self.n_layers)
            return InitConfig(in_std=in_std, attn_out_std=out_std, ff_out_std=out_std)
        raise NotImplementedError(self.init_type)


def rms_norm_reference(x: Tensor, eps: float) -> Tensor:
    return F.rms_norm(x.float(), (x.shape[-1],), eps=eps).to(x.dtype)


class TransformerBlock(nn.Module):
    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.norm_type = config.norm_type
        self.norm_eps = config.norm_eps
        self.attn = Attention(hidden_size=config.hidden_size, head_dim=config.head_dim,
                              num_heads=config.num_heads, num_key_value_heads=config.num_heads,
                              attn_type=config.attn_type, init_std_in=config.init_config.in_std,
                              init_std_out=config.init_config.attn_out_std)
        self.mlp = SwiGLU(hidden_size=config.hidden_size, intermediate_size=config.intermediate_size,
                          init_std_in=config.init_config.in_std, init_std_out=config.init_config.ff_out_std)

    def norm(self, x: Tensor) -> Tensor:
        return rms_norm_reference(x, self.norm_eps)

    def forward(self, x: Tensor, **seq_info) -> Tensor:
        if self.norm_type == "pre":
            x = x + self.attn(self.norm(x), **seq_info)
            return x + self.mlp(self.norm(x))
        x = self.norm(x + self.attn(x, **seq_info))
        return self.norm(x + self.mlp(x))


class Transformer(nn.Module):
    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.config = config
        self.head_hint = {"in": {"dim": config.hidden_size, "init_std": config.init_config.in_std},
                          "out": {"dim": config.hidden_size, "init_std": config.init_config.in_std}}
        if config.pos_emb_type == "rope":
            assert config.rope_theta is not None
            self.rotary_emb = RotaryEmbedding(config.head_dim, config.max_seq_len, base=config.rope_theta)
        self.layers = nn.ModuleList([TransformerBlock(config) for _ in range(config.n_layers)])

    def create_cache(self, **kwargs) -> list[Cache]:
        return [Cache.create(**kwargs, num_heads=self.config.num_heads, head_dim=self.config.head_dim)
                for _ in range(self.config.n_layers)]

    def final_norm(self, x: Tensor) -> Tensor:
        return rms_norm_reference(x, self.config.norm_eps) if self.config.norm_type == "pre" else x

    def forward(self, x: Tensor, cache: Optional[list[Cache]] = None, injection: Optional[Tensor] = None,
                **seq_info) -> Tensor:
        """Run the stack on ``x (+ injection)``; ``seq_info`` carries packing metadata."""
        if fused_path(x if injection is None else injection):
            from ..ops import block as fused_block
            if cache is None:
                return fused_block.stack_forward(self, x, injection, seq_info)
            if not torch.is_grad_enabled() and seq_info.get("position_ids") is not None:
                out = fused_block.stack_forward_cached(self, x, injection, cache, seq_info.get("cache_lengths"),
                                                       seq_info["position_ids"])
                if out is not None:
                    return out

        if injection is not None:
            x = x + injection
        position_ids = seq_info.pop("position_ids", None)
        cos_sin = self.rotary_emb(position_ids) if hasattr(self, "rotary_emb") else None
        for i, layer in enumerate(self.layers):
            x = layer(x, cos_sin=cos_sin, cache=cache[i] if cache is not None else None, **seq_info)
        return self.final_norm(x)
