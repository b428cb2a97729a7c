"""KV-cache attention on sm_100a kernels for inference.

* ``kv_decode``: one new token per sequence (the decode step). Appends the token's key and
  value at ``cache_lengths`` and attends over ``[0, cache_lengths + 1)`` with the split-KV
  decode kernel (csrc/kernels/decode.cu).
* ``kv_prefill``: a whole prompt into an empty cache (the prefill step, one sequence). Writes
  the prompt's keys and values into the cache and runs the tcgen05 PrefixLM kernel over the
  prompt (bidirectional, or causal when the layer is causal).

Both match ``models.layers.cached_attention_reference`` (reference models/layers.py:148-151,
``flash_attn_with_kvcache`` with ``cache_seqlens``) for the cases the inference engine issues.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .._native import cuda


def kv_decode(query: Tensor, key: Tensor, value: Tensor, cache, cache_lengths: Tensor) -> Tensor:
    """``query, key, value: [B, 1, H, 128]``; ``cache_lengths: [B]``. Returns ``[B, 1, H, 128]``."""
    bsz = query.shape[0]
    lengths = cache_lengths.to(device=query.device, dtype=torch.long).reshape(-1)
    rows = torch.arange(bsz, device=query.device)
    cache.keys[rows, lengths] = key[:, 0].to(cache.keys.dtype)
    cache.values[rows, lengths] = value[:, 0].to(cache.values.dtype)
    total = (lengths + 1).to(torch.int32)
    out = cuda().decode_attention(query[:, 0].contiguous(), cache.keys, cache.values, total)
    return out[:, None]


def kv_prefill(query: Tensor, key: Tensor, value: Tensor, cache, is_causal: bool) -> Tensor:
    """``query, key, value: [1, L, H, 128]`` into an empty cache. Returns ``[1, L, H, 128]``."""
    from .attention import flash_attn_varlen_prefixlm
    L = query.shape[1]
    cache.keys[0, :L] = key[0].to(cache.keys.dtype)
    cache.values[0, :L] = value[0].to(cache.values.dtype)
    dev = query.device
    cu = torch.tensor([0, L], dtype=torch.int32, device=dev)
    prefix = torch.tensor([0 if is_causal else L], dtype=torch.int32, device=dev)
    out = flash_attn_varlen_prefixlm(query[0].contiguous(), key[0].contiguous(), value[0].contiguous(), is_causal,
                                     prefix, None, cu)
    return out[None]
