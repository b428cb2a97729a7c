"""PrefixLM packed-varlen attention on the device (csrc/kernels/attention.cu).

``PackedSeq`` carries one step's packing metadata (token positions, ``cu_seqlens``,
per-document prefix lengths) and lazily builds the device-side work schedule that the
attention kernels consume. The schedule is computed on the GPU from ``cu_seqlens`` alone,
so the whole step can be captured in a CUDA graph and replayed with new batches.

``flash_attn_varlen_prefixlm`` keeps the reference's call signature
(models/flash_attention_prefixlm_v2.py:271-282) for code that calls attention directly on
separate q, k, v tensors.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor

from .._native import cuda


class PackedSeq:
    """Device metadata of one packed batch of ``T`` tokens."""

    def __init__(self, position_ids: Tensor, cu_seqlens: Tensor, prefix_lens: Tensor):
        self.position_ids = position_ids.to(torch.int32).contiguous()
        self.cu_seqlens = cu_seqlens.to(torch.int32).contiguous()
        self.prefix_lens = prefix_lens.to(torch.int32).contiguous()
        self.T = int(self.position_ids.numel())
        self._sched: dict[bool, Tensor] = {}

    def schedule(self, causal: bool) -> Tensor:
        sched = self._sched.get(causal)
        if sched is None:
            cap = cuda().attn_schedule_capacity(self.T, self.cu_seqlens.numel())
            sched = torch.empty(8 + 8 * cap, dtype=torch.int32, device=self.cu_seqlens.device)
            cuda().attn_schedule(self.cu_seqlens, self.prefix_lens, causal, self.T, sched)
            self._sched[causal] = sched
        return sched

    @staticmethod
    def from_seq_info(seq_info: dict) -> "PackedSeq":
        packed = seq_info.get("packed")
        if packed is None:
            packed = PackedSeq(seq_info["position_ids"], seq_info["cu_seqlens"], seq_info["prefix_lens"])
            seq_info["packed"] = packed
        return packed


def rope_half_tables(module: torch.nn.Module) -> tuple[Tensor, Tensor]:
    """fp32 ``[max_seq_len, head_dim/2]`` cos/sin tables derived from a ``RotaryEmbedding``."""
    tabs = getattr(module, "_half_tables", None)
    cos = module.cos_cached
    if tabs is None or tabs[0].device != cos.device:
        half = cos.shape[-1] // 2
        tabs = (cos[:, :half].float().contiguous(), module.sin_cached[:, :half].float().contiguous())
        module._half_tables = tabs
    return tabs


def attention_fwd(gqkv: Tensor, num_heads: int, sched: Tensor, kernel: str = "tcgen05"):
    """Returns ``(O, Y = sigmoid(gate) * O, lse)`` for the packed ``gqkv [T, 4*H*128]``.

    ``kernel="tcgen05"`` (training path) runs the TMEM/UMMA kernel (attention_tc.cu);
    ``kernel="mma"`` runs the warp-level mma.sync kernel (attention.cu), kept as a
    cross-check.
    """
    T = gqkv.shape[0]
    width = num_heads * 128
    out = torch.empty((T, width), dtype=torch.bfloat16, device=gqkv.device)
    y = torch.empty_like(out)
    lse = torch.empty((num_heads, T), dtype=torch.float32, device=gqkv.device)
    if kernel == "tcgen05":
        cuda().attn_fwd_tc(gqkv, num_heads, sched, out, y, lse)
    else:
        cuda().attn_fwd(gqkv, num_heads, sched, out, y, lse)
    return out, y, lse


def attention_bwd(gqkv: Tensor, num_heads: int, sched: Tensor, out: Tensor, lse: Tensor, dy: Tensor,
                  positions: Tensor, cos: Tensor, sin: Tensor, kernel: str = "tcgen05") -> Tensor:
    """Gradient w.r.t. the packed ``gqkv`` (gate, q, k, v; RoPE backward applied to q, k).

    ``kernel="tcgen05"`` runs the TMEM/UMMA backward (attention_tc.cu); ``"mma"`` the
    mma.sync backward (attention.cu), kept as a cross-check.
    """
    T = gqkv.shape[0]
    width = num_heads * 128
    d_out = torch.empty((T, width), dtype=torch.bfloat16, device=gqkv.device)
    dsum = torch.empty((num_heads, T), dtype=torch.float32, device=gqkv.device)
    dq_acc = torch.empty((T, width), dtype=torch.float32, device=gqkv.device)
    dgqkv = torch.empty((T, 4 * width), dtype=torch.bfloat16, device=gqkv.device)
    fn = cuda().attn_bwd_tc if kernel == "tcgen05" else cuda().attn_bwd
    fn(gqkv, num_heads, sched, out, lse, dy, positions, cos, sin, d_out, dsum, dq_acc, dgqkv)
    return dgqkv


BWD_PHASES = ("wait S", "softmax math", "wait P free", "store P/dS", "wait dQ", "drain dQ", "dK/dV epilogue",
              "other (compute warp)", "MMA wait Q/dO", "MMA wait dQ free", "MMA issue S/dP", "MMA wait P",
              "MMA wait dK/dV free", "MMA issue dV/dK/dQ + other", "MMA wait K/V", "query blocks",
              "epilogue wait dK/dV", "epilogue work", "item fetch", "unused")


def bwd_phase_profile(fn) -> dict:
    """Run ``fn`` with phase tracing of the tcgen05 backward enabled and return the cycles per
    phase (one compute warp and the UMMA thread of every CTA, summed over CTAs) plus the number
    of query blocks the traced warps processed."""
    c = cuda()
    c.attn_bwd_phase_counters(True)
    c.attn_bwd_set_profile(True)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        c.attn_bwd_set_profile(False)
    vals = c.attn_bwd_phase_counters(True).tolist()
    return dict(zip(BWD_PHASES, vals))


class _VarlenPrefixLM(torch.autograd.Function):
    """Attention on separate (already rotated) q, k, v; used by the compatibility API."""

    @staticmethod
    def forward(ctx, q, k, v, is_causal, packed: PackedSeq):
        T, H, D = q.shape
        assert D == 128, "the sm_100a attention kernels are specialised for head_dim 128"
        gate = torch.full_like(q, 30.0)  # sigmoid(30) == 1 in fp32: Y == O
        gqkv = torch.cat([gate, q, k, v], dim=1).reshape(T, 4 * H * D).contiguous()
        sched = packed.schedule(bool(is_causal))
        out, _, lse = attention_fwd(gqkv, H, sched)
        ctx.save_for_backward(gqkv, out, lse)
        ctx.packed, ctx.causal, ctx.H = packed, bool(is_causal), H
        return out.view(T, H, D)

    @staticmethod
    def backward(ctx, dout):
        gqkv, out, lse = ctx.saved_tensors
        packed, H = ctx.packed, ctx.H
        T = gqkv.shape[0]
        # identity rotation: positions 0 with cos=1, sin=0
        zeros = torch.zeros(T, dtype=torch.int32, device=gqkv.device)
        cos = torch.ones((1, 64), dtype=torch.float32, device=gqkv.device)
        sin = torch.zeros((1, 64), dtype=torch.float32, device=gqkv.device)
        dg = attention_bwd(gqkv, H, packed.schedule(ctx.causal), out, lse, dout.reshape(T, H * 128).contiguous(),
                           zeros, cos, sin).view(T, 4, H, 128)
        return dg[:, 1], dg[:, 2], dg[:, 3], None, None


def flash_attn_varlen_prefixlm(q: Tensor, k: Tensor, v: Tensor, is_causal: bool, prefix_lens: Tensor,
                               causal_lens: Optional[Tensor], cu_seqlens: Tensor, total_seqlen=None, numseqs=None,
                               max_seqlen_prefix=None, max_seqlen_causal=None, max_seqlen_all=None,
                               position_ids: Optional[Tensor] = None) -> Tensor:
    """PrefixLM varlen attention with the reference's signature; host scalars are optional."""
    T = q.shape[0]
    pos = position_ids if position_ids is not None else torch.zeros(T, dtype=torch.int32, device=q.device)
    packed = PackedSeq(pos, cu_seqlens, prefix_lens)
    return _VarlenPrefixLM.apply(q, k, v, is_causal, packed)


def softmax_scale(head_dim: int = 128) -> float:
    return 1.0 / math.sqrt(head_dim)
