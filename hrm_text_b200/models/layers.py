"""Neural-network layers of HRM-Text with the reference's parameter names.

Parameter names, shapes and init match reference models/layers.py so checkpoints are
interchangeable:
* ``LinearInit.weight`` is ``[prod(batch_out_features) * out_features, in_features]``,
  truncated-LeCun init (layers.py:61-85);
* ``ScaledEmbeddingInit.embedding_weight`` is ``[V, h]`` and the output is multiplied by
  ``1/init_std`` (layers.py:88-102);
* ``Attention.gqkv_proj`` packs gate, q, k, v heads in that order (layers.py:116-155);
* ``SwiGLU.gate_up_proj`` packs gate rows first, then up rows (layers.py:158-168).

The modules here are the *CPU oracle* path: plain torch, fp32-capable, autograd. On CUDA the
Transformer stack does not call these ``forward`` methods; it runs the fused sm_100a block
(``hrm_text_b200.ops.block``) on the same parameters.
"""
from __future__ import annotations

import math
from typing import NamedTuple, Optional, Sequence

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .common import trunc_normal_init_


def find_multiple(a: int, b: int) -> int:
    """Smallest multiple of ``b`` that is >= ``a``."""
    return ((a + b - 1) // b) * b


def rope_tables(head_dim: int, max_seq_len: int, base: float, device=None) -> tuple[Tensor, Tensor]:
    """fp32 cos/sin tables ``[max_seq_len, head_dim]`` in rotate-half layout.

    Frequency ``i`` (``0 <= i < head_dim/2``) is ``base ** (-2i/head_dim)``; columns ``i`` and
    ``i + head_dim/2`` share it, which is the layout the rotate-half formulation expects.
    """
    half = head_dim // 2
    inv_freq = torch.pow(torch.tensor(float(base), dtype=torch.float32, device=device),
                         -torch.arange(0, half, dtype=torch.float32, device=device) * (2.0 / head_dim))
    angles = torch.arange(max_seq_len, dtype=torch.float32, device=device)[:, None] * inv_freq[None, :]
    angles = torch.cat([angles, angles], dim=-1)
    return angles.cos(), angles.sin()


def rotate_half(x: Tensor) -> Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary_pos_emb(x: Tensor, cos_sin: tuple[Tensor, Tensor]) -> Tensor:
    """RoPE in fp32 on ``x [..., S, heads, head_dim]`` with ``cos, sin [..., S, head_dim]``."""
    cos, sin = cos_sin
    xf = x.float()
    return (xf * cos.unsqueeze(-2) + rotate_half(xf) * sin.unsqueeze(-2)).to(x.dtype)


class RotaryEmbedding(nn.Module):
    """Holds non-persistent cos/sin caches (``cos_cached``, ``sin_cached``)."""

    def __init__(self, dim: int, max_seq_len: int, base: float, device=None):
        super().__init__()
        cos, sin = rope_tables(dim, max_seq_len, base, device=device)
        self.cos_cached = nn.Buffer(cos, persistent=False)
        self.sin_cached = nn.Buffer(sin, persistent=False)

    def forward(self, position_ids: Optional[Tensor]):
        if position_ids is None:
            return self.cos_cached, self.sin_cached
        ids = position_ids.long()
        return self.cos_cached[ids], self.sin_cached[ids]


class LinearInit(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool,
                 batch_out_features: Sequence[int] = (), init_std: Optional[float] = None, **kwargs):
        super().__init__()
        self.in_features = in_features
        std = init_std if init_std is not None else 1.0 / math.sqrt(in_features)
        rows = math.prod(batch_out_features) * out_features
        self.weight = nn.Parameter(trunc_normal_init_(torch.empty((rows, in_features), **kwargs), std=std))
        self.bias = nn.Parameter(torch.zeros((rows,), **kwargs)) if bias else None

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))


class ScaledEmbeddingInit(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int, init_std: float, **kwargs):
        super().__init__()
        self.scale = 1.0 / init_std
        self.embedding_weight = nn.Parameter(
            trunc_normal_init_(torch.empty((num_embeddings, embedding_dim), **kwargs), std=init_std))

    def forward(self, ids: Tensor) -> Tensor:
        return self.scale * F.embedding(ids.long(), self.embedding_weight)


class Cache(NamedTuple):
    """Static KV cache of one attention layer: ``[B, S_max, heads, head_dim]`` each."""

    keys: Tensor
    values: Tensor

    @classmethod
    def create(cls, max_batch_size: int, max_seq_len: int, num_heads: int, head_dim: int, **kwargs):
        shape = (max_batch_size, max_seq_len, num_heads, head_dim)
        return cls(keys=torch.zeros(shape, **kwargs), values=torch.zeros(shape, **kwargs))


def prefixlm_allowed(doc_len: int, prefix_len: int, device=None) -> Tensor:
    """Boolean ``[doc_len, doc_len]`` mask: query ``i`` sees key ``j`` iff ``j < max(prefix_len, i+1)``.

    This is the union of the reference's two FlashAttention passes
    (flash_attention_prefixlm_v2.py:115-131): bidirectional inside the prefix, and
    bottom-right-aligned causal for response queries against the whole document.
    """
    i = torch.arange(doc_len, device=device)
    limit = torch.clamp(i + 1, min=prefix_len)
    return torch.arange(doc_len, device=device)[None, :] < limit[:, None]


def doc_boundaries(cu_seqlens: Tensor) -> list[tuple[int, int, int]]:
    """``[(doc_index, start, end)]`` for a padded ``cu_seqlens`` (stops at the zero padding)."""
    cu = cu_seqlens.tolist()
    out = []
    for i in range(len(cu) - 1):
        if cu[i + 1] <= cu[i]:
            break
        out.append((i, cu[i], cu[i + 1]))
    return out


def prefixlm_attention_reference(q: Tensor, k: Tensor, v: Tensor, is_causal: bool,
                                 prefix_lens: Tensor, cu_seqlens: Tensor) -> Tensor:
    """Packed varlen PrefixLM attention in fp32 (the CPU oracle). ``q,k,v: [T, heads, d]``.

    Rows outside every document (the padding tail) are zero.
    """
    out = torch.zeros_like(q)
    scale = 1.0 / math.sqrt(q.shape[-1])
    prefixes = prefix_lens.tolist()
    for d, start, end in doc_boundaries(cu_seqlens):
        p = 0 if is_causal else prefixes[d]
        mask = prefixlm_allowed(end - start, p, device=q.device)
        qd, kd, vd = (t[start:end].float().transpose(0, 1) for t in (q, k, v))
        o = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=mask, scale=scale)
        out[start:end] = o.transpose(0, 1).to(q.dtype)
    return out


def cached_attention_reference(q: Tensor, k: Tensor, v: Tensor, cache: Cache, cache_lengths,
                               is_causal: bool) -> Tensor:
    """Attention against a static KV cache, after appending ``k, v`` at ``cache_lengths``.

    ``q, k, v: [B, S, heads, d]``; ``cache_lengths``: int or ``[B]`` tensor. New keys are
    written in place into ``cache``. Query ``s`` of row ``b`` sees cache positions
    ``< cache_lengths[b] + S`` (all of them when not causal; up to its own position when
    causal), matching a KV-cache attention call with ``cache_seqlens`` semantics.
    """
    bsz, seq = q.shape[0], q.shape[1]
    if isinstance(cache_lengths, int):
        lengths = torch.full((bsz,), cache_lengths, dtype=torch.long, device=q.device)
    else:
        lengths = cache_lengths.to(device=q.device, dtype=torch.long).reshape(-1)
    pos = lengths[:, None] + torch.arange(seq, device=q.device)[None, :]
    batch_idx = torch.arange(bsz, device=q.device)[:, None].expand(bsz, seq)
    cache.keys[batch_idx, pos] = k.to(cache.keys.dtype)
    cache.values[batch_idx, pos] = v.to(cache.values.dtype)
    total = lengths + seq
    kpos = torch.arange(cache.keys.shape[1], device=q.device)
    mask = kpos[None, None, :] < total[:, None, None]
    if is_causal:
        mask = mask & (kpos[None, None, :] <= pos[:, :, None])
    else:
        mask = mask.expand(bsz, seq, kpos.shape[0])
    scale = 1.0 / math.sqrt(q.shape[-1])
    o = F.scaled_dot_product_attention(q.float().transpose(1, 2), cache.keys.float().transpose(1, 2),
                                       cache.values.float().transpose(1, 2), attn_mask=mask[:, None],
                                       scale=scale)
    return o.transpose(1, 2).to(q.dtype)


def cached_attention(q: Tensor, k: Tensor, v: Tensor, cache: Cache, cache_lengths, is_causal: bool) -> Tensor:
    """KV-cache attention: the sm_100a kernels for the decode step (one token per sequence)
    and for a prompt prefilled into an empty cache; the torch reference for anything else
    (CPU, other dtypes or head sizes, multi-token appends to a non-empty cache)."""
    fast = q.is_cuda and q.shape[-1] == 128 and q.dtype == torch.bfloat16 and cache.keys.dtype == torch.bfloat16
    if fast and q.shape[1] == 1 and not isinstance(cache_lengths, int):
        from ..ops.decode import kv_decode
        return kv_decode(q, k, v, cache, cache_lengths)
    if fast and isinstance(cache_lengths, int) and cache_lengths == 0 and q.shape[0] == 1:
        from ..ops.decode import kv_prefill
        return kv_prefill(q, k, v, cache, is_causal)
    return cached_attention_reference(q, k, v, cache, cache_lengths, is_causal)


class Attention(nn.Module):
    def __init__(self, hidden_size: int, head_dim: int, num_heads: int, num_key_value_heads: int,
                 attn_type: str, init_std_in=None, init_std_out=None, **kwargs):
        super().__init__()
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.num_key_value_heads = num_key_value_heads
        self.attn_type = attn_type
        self.gqkv_proj = LinearInit(hidden_size, head_dim, bias=False,
                                    batch_out_features=(2 * num_heads + 2 * num_key_value_heads,),
                                    init_std=init_std_in, **kwargs)
        self.o_proj = LinearInit(head_dim * num_heads, hidden_size, bias=False, init_std=init_std_out, **kwargs)

    def split_gqkv(self, gqkv: Tensor):
        shape = gqkv.shape[:-1] + (2 * self.num_heads + 2 * self.num_key_value_heads, self.head_dim)
        heads = gqkv.view(shape)
        return heads.split((self.num_heads, self.num_heads, self.num_key_value_heads, self.num_key_value_heads), dim=-2)

    def forward(self, hidden_states: Tensor, cos_sin=None, cache: Optional[Cache] = None,
                cache_lengths=None, prefix_lens: Optional[Tensor] = None,
                cu_seqlens: Optional[Tensor] = None, **unused) -> Tensor:
        gate, query, key, value = self.split_gqkv(self.gqkv_proj(hidden_states))
        if cos_sin is not None:
            query = apply_rotary_pos_emb(query, cos_sin)
            key = apply_rotary_pos_emb(key, cos_sin)
        is_causal = self.attn_type == "causal"
        if cache is None:
            attn = prefixlm_attention_reference(query, key, value, is_causal, prefix_lens, cu_seqlens)
        else:
            attn = cached_attention(query, key, value, cache, cache_lengths, is_causal)
        gated = torch.sigmoid(gate.float()).to(attn.dtype) * attn
        return self.o_proj(gated.flatten(-2))


class SwiGLU(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int, init_std_in=None, init_std_out=None, **kwargs):
        super().__init__()
        self.gate_up_proj = LinearInit(hidden_size, intermediate_size, bias=False, batch_out_features=(2,),
                                       init_std=init_std_in, **kwargs)
        self.down_proj = LinearInit(intermediate_size, hidden_size, bias=False, init_std=init_std_out, **kwargs)

    def forward(self, x: Tensor) -> Tensor:
        gate, up = self.gate_up_proj(x).chunk(2, dim=-1)
        return self.down_proj(F.silu(gate) * up)
