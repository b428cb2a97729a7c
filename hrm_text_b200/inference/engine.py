"""Inference: checkpoint loading and batched generation with static KV caches.

Behaviour follows the reference's simple_inference_engine.py:
* ``inference_load_checkpoint`` (:37-90) rebuilds the model from ``all_config.yaml`` /
  ``train_metadata.yaml``, loads the DCP checkpoint on one process, optionally swaps in the EMA
  weights, casts to the forward dtype and loads the tokenizer;
* ``inference_generate`` (:115-197) is a generator doing continuous batching over
  ``batch_size`` slots: a free slot is filled by a bidirectional prefill of one prompt (the
  PrefixLM prefix), then all active slots decode one token per step; finished generations are
  yielded as ``(prompt_id, text)``; prompts that do not fit the context yield ``""``;
* sampling is greedy for ``temp < 1e-5`` and Gumbel-max otherwise (:93-102).

Every module call of the recurrent model has its own static cache (one per call and layer,
``model.create_cache``).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Generator, Iterator, Optional

import numpy as np
import torch
from torch import Tensor, nn

from ..config import PretrainConfig
from ..data.dataset import V1DatasetMeta
from ..optim.adam_atan2 import AdamATan2
from ..runtime.checkpoint import checkpoint_dir, latest_epoch
from ..runtime.factory import build_model, model_config_dict


@dataclass
class InferenceCheckpoint:
    model: nn.Module
    carry: Any
    tokenizer: Any
    tokenizer_info: dict

    def tokenize_prompt(self, condition: str, prompt: str) -> np.ndarray:
        info = self.tokenizer_info
        cond = "".join(info["condition_mapping"][c] for c in condition.split(","))
        text = f'{info["boq"]}{cond}{prompt}{info["eoq"]}'
        return np.asarray(self.tokenizer(text, add_special_tokens=False)["input_ids"], dtype=np.int64)

    def decode_generation(self, tokens: np.ndarray, eos_id: int) -> str:
        if tokens.size and tokens[-1] == eos_id:
            tokens = tokens[:-1]
        return self.tokenizer.decode(tokens.tolist())


def load_model_from_checkpoint(ckpt_path: str, ckpt_epoch: Optional[int] = None, use_ema: bool = True,
                               device: Optional[torch.device] = None):
    """Model (eval mode, forward dtype) + carry + metadata, from a training checkpoint directory."""
    import yaml
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict
    device = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                        else torch.device("cpu"))
    with open(os.path.join(ckpt_path, "all_config.yaml")) as f:
        cfg = PretrainConfig(**yaml.safe_load(f))
    with open(os.path.join(ckpt_path, "train_metadata.yaml")) as f:
        meta = V1DatasetMeta(**yaml.safe_load(f))
    model_cfg = model_config_dict(cfg.arch.model_dump(), meta.model_dump(), cfg.data.model_dump())
    model = build_model(model_cfg, device)
    optim = AdamATan2(model.parameters(), lr=torch.tensor(0.0), betas=(cfg.beta1, cfg.beta2),
                      weight_decay=cfg.weight_decay, ema=cfg.ema)
    if ckpt_epoch is None:
        ckpt_epoch = latest_epoch(ckpt_path)
        if ckpt_epoch is None:
            raise ValueError(f"No checkpoint files found in {ckpt_path}")
    dcp.load({"model": model.state_dict(), "optim": get_optimizer_state_dict(model, optim)},
             checkpoint_id=checkpoint_dir(ckpt_path, ckpt_epoch), no_dist=True)
    carry_file = os.path.join(ckpt_path, f"carry_epoch_{ckpt_epoch}.0.pt")
    carry = torch.load(carry_file, map_location=device, weights_only=False) if os.path.exists(carry_file) else None
    if use_ema:
        optim.swap_ema()
    model = model.to(getattr(torch, cfg.fwd_bwd_dtype)).eval()
    return model, carry, cfg, meta


def inference_load_checkpoint(ckpt_path: str, ckpt_epoch: Optional[int], ckpt_use_ema: bool) -> InferenceCheckpoint:
    from transformers import AutoTokenizer
    model, carry, _cfg, meta = load_model_from_checkpoint(ckpt_path, ckpt_epoch, ckpt_use_ema)
    tokenizer = AutoTokenizer.from_pretrained(meta.tokenizer_info["tokenizer_path"], use_fast=True)
    return InferenceCheckpoint(model=model, carry=carry, tokenizer=tokenizer, tokenizer_info=meta.tokenizer_info)


_SAMPLE_CALLS = [0]


def sample(logits: Tensor, temp: float, generator: Optional[torch.Generator] = None) -> Tensor:
    """Greedy for ``temp < 1e-5``; else Gumbel-max sampling at temperature ``temp``.

    On CUDA one fused kernel does the scaling, the Gumbel noise (counter-based, seeded from
    ``generator`` or torch's default seed, advanced every call) and the argmax.
    """
    if logits.is_cuda and logits.dim() == 2 and logits.dtype in (torch.float32, torch.bfloat16):
        from .._native import cuda
        seed = generator.initial_seed() if generator is not None else torch.initial_seed()
        _SAMPLE_CALLS[0] += 1
        return cuda().sample_tokens(logits.contiguous(), float(temp), int(seed) & 0x7FFFFFFFFFFFFFFF, _SAMPLE_CALLS[0])
    if temp < 1e-5:
        return logits.argmax(-1)
    scaled = logits.float() / temp
    u = torch.rand(scaled.shape, device=scaled.device, generator=generator).clamp_min(torch.finfo(torch.float32).tiny)
    return (scaled - torch.log(-torch.log(u))).argmax(-1)


@torch.inference_mode()
def prefill(model: nn.Module, carry, tokens: Tensor, cache) -> Tensor:
    """Bidirectional pass over one prompt into ``cache``; returns the last position's logits."""
    batch = {"inputs": tokens[None], "position_ids": torch.arange(tokens.numel(), device=tokens.device),
             "cache": cache, "cache_lengths": 0}
    return model(carry=carry, batch=batch)[-1][0, -1]


@torch.inference_mode()
def decode_step(model: nn.Module, carry, last_tokens: Tensor, cache, cache_lengths: Tensor) -> Tensor:
    batch = {"inputs": last_tokens[:, None], "position_ids": cache_lengths[:, None], "cache": cache,
             "cache_lengths": cache_lengths}
    return model(carry=carry, batch=batch)[-1][:, -1]


class DecodeGraph:
    """The decode step (all ``batch_size`` slots, one token each) captured in one CUDA graph.

    The step's work is a fixed sequence of device operations on static shapes (embedding,
    per module call and layer the RMSNorm / GEMM / decode-attention kernels, the LM-head GEMM),
    so it is captured once per cache and replayed for every generated token; the per-step
    inputs (last tokens, cache lengths) are copied into static buffers. Capture writes junk
    keys / values at position 0 of every slot, so it must happen before any prompt is
    prefilled into the cache.
    """

    def __init__(self, model: nn.Module, carry, cache, batch_size: int, device: torch.device, warmup: int = 2):
        self.tokens = torch.zeros(batch_size, dtype=torch.long, device=device)
        self.lengths = torch.zeros(batch_size, dtype=torch.int32, device=device)
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                decode_step(model, carry, self.tokens, cache, self.lengths)
        torch.cuda.current_stream(device).wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.logits = decode_step(model, carry, self.tokens, cache, self.lengths)

    def __call__(self, last_tokens: Tensor, cache_lengths: Tensor) -> Tensor:
        self.tokens.copy_(last_tokens, non_blocking=True)
        self.lengths.copy_(cache_lengths, non_blocking=True)
        self.graph.replay()
        return self.logits


def _slot_view(cache, i: int):
    return torch.utils._pytree.tree_map(lambda x: x[i:i + 1] if isinstance(x, Tensor) else x, cache)


@torch.inference_mode()
def generate_tokens(model: nn.Module, carry, prompts: Iterator[tuple[int, np.ndarray]], max_tokens: int,
                    max_generation: int, batch_size: int, stop_token: int, temp: float = 0.0,
                    device: Optional[torch.device] = None,
                    use_cuda_graph: bool = True) -> Generator[tuple[int, np.ndarray], None, None]:
    """Continuous-batching generation over token prompts; yields ``(prompt_id, generated_ids)``.

    On a CUDA device with bf16 weights the decode step runs as one captured CUDA graph
    (``DecodeGraph``)."""
    device = device or next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    cache = model.create_cache(max_batch_size=batch_size, max_seq_len=max_tokens, dtype=dtype, device=device)
    graphed = None
    if use_cuda_graph and device.type == "cuda" and dtype == torch.bfloat16:
        graphed = DecodeGraph(model, carry, cache, batch_size, device)  # before any prefill (see DecodeGraph)
    lengths = torch.zeros(batch_size, dtype=torch.int32, device=device)
    last = torch.zeros(batch_size, dtype=torch.long, device=device)
    generated = np.zeros((batch_size, max_tokens), dtype=np.int64)
    g_start = np.zeros(batch_size, dtype=np.int64)
    g_len = np.zeros(batch_size, dtype=np.int64)
    stopped = np.ones(batch_size, dtype=bool)
    ids = [-1] * batch_size

    def next_prompt():
        for pid, tok in prompts:
            if tok.size >= max_tokens:
                yield pid, np.zeros(0, dtype=np.int64)
                continue
            return pid, tok
        return -1, None

    pending_id, pending = yield from next_prompt()
    while True:
        for i in np.nonzero(stopped)[0]:
            if ids[i] != -1:
                yield ids[i], generated[i, g_start[i]:g_len[i]].copy()
                ids[i] = -1
            if pending is None:
                continue
            tok = torch.as_tensor(pending, device=device)
            logits = prefill(model, carry, tok, _slot_view(cache, int(i)))
            first = int(sample(logits[None], temp)[0])
            lengths[i] = pending.size
            last[i] = first
            ids[i] = pending_id
            g_start[i] = max(pending.size, max_tokens - max_generation)
            g_len[i] = g_start[i] + 1
            generated[i, g_start[i]] = first
            stopped[i] = first == stop_token or g_len[i] >= max_tokens
            pending_id, pending = yield from next_prompt()
        if not stopped.all():
            logits = graphed(last, lengths) if graphed is not None else decode_step(model, carry, last, cache, lengths)
            last = sample(logits, temp)
            lengths.add_(1).clamp_max_(max_tokens - 1)
            active = ~stopped
            g_len[active] += 1
            host = last.cpu().numpy()
            generated[active, g_len[active] - 1] = host[active]
            stopped |= (host == stop_token) | (g_len >= max_tokens)
        elif pending is None:
            break
    for i in range(batch_size):
        if ids[i] != -1:
            yield ids[i], generated[i, g_start[i]:g_len[i]].copy()


def inference_generate(ckpt: InferenceCheckpoint, iterator: Iterator[tuple[int, tuple[str, str]]], max_tokens: int,
                       max_generation: int, batch_size: int, temp: float = 0.0) -> Generator[tuple[int, str], None, None]:
    """Text in, text out: ``iterator`` yields ``(prompt_id, (condition, prompt))``."""
    stop = ckpt.tokenizer.convert_tokens_to_ids(ckpt.tokenizer_info["eoa"])
    tokenized = ((pid, ckpt.tokenize_prompt(*p)) for pid, p in iterator)
    for pid, toks in generate_tokens(ckpt.model, ckpt.carry, tokenized, max_tokens, max_generation, batch_size,
                                     stop, temp):
        yield pid, ckpt.decode_generation(toks, stop) if toks.size else ""
