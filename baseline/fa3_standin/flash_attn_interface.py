"""Stand-in for FlashAttention-3's ``flash_attn_interface`` on B200 (reference arm only).

FlashAttention-3 (the reference's attention, built from ``hopper/``) is sm_90a-only and is
not installed here. The reference's PrefixLM op (models/flash_attention_prefixlm_v2.py) calls
three things from it; this module provides them with FA3's varlen semantics, implemented on
FlashAttention-2 (``flash_attn`` 2.8, sm_80+ kernels) or, if FA2 cannot run, on PyTorch SDPA:

* ``torch.ops.flash_attn_3.fwd(q, k, v, ..., out, cu_seqlens_q, cu_seqlens_k, seqused_q,
  seqused_k, max_seqlen_q, max_seqlen_k, ..., is_causal, ...)`` -> ``(out, softmax_lse, ...)``;
  rows outside the used ranges are left untouched in ``out`` (the reference runs two passes
  into one buffer);
* ``_flash_attn_backward(dout, q, k, v, out, softmax_lse, cu_seqlens_q, cu_seqlens_k,
  max_seqlen_q, max_seqlen_k, sequed_q, sequed_k, dq, dk, dv, is_causal)`` writing the used
  rows of ``dq`` / ``dk`` / ``dv``;
* ``flash_attn_with_kvcache`` and ``maybe_contiguous``.

FA3's ``seqused_*`` (only the first ``seqused[i]`` rows of item ``i`` are used) has no FA2
equivalent for queries, so used rows are gathered into a packed tensor on the device
(stable ordering through an argsort of the "unused" mask: no host sync), run through FA2
varlen (bottom-right-aligned causal mask, as FA3), and scattered back. Nothing here is part
of the HRM-Text B200 framework; it only lets the unmodified reference run on this GPU.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

BACKEND = os.environ.get("HRM_REF_ATTN_BACKEND", "fa2")
_fa2 = None


def _fa2_module():
    global _fa2, BACKEND
    if _fa2 is None and BACKEND == "fa2":
        try:
            from flash_attn import flash_attn_interface as fa2
            _fa2 = fa2
        except Exception:  # pragma: no cover
            BACKEND = "sdpa"
    return _fa2


def maybe_contiguous(x):
    return x.contiguous() if x is not None and x.stride(-1) != 1 else x


def _used_rows(cu: torch.Tensor, used: Optional[torch.Tensor], total: int):
    """Mask of rows in ``[cu[i], cu[i] + used[i])`` and packed cu of the used rows (device only)."""
    cu = cu.to(torch.int64)
    lens = (cu[1:] - cu[:-1]) if used is None else used.to(torch.int64)
    marks = torch.zeros(total + 1, dtype=torch.int64, device=cu.device)
    marks.index_add_(0, cu[:-1].clamp(max=total), torch.ones_like(lens))
    marks.index_add_(0, (cu[:-1] + lens).clamp(max=total), -torch.ones_like(lens))
    mask = marks.cumsum(0)[:total] > 0
    packed_cu = torch.zeros(lens.numel() + 1, dtype=torch.int32, device=cu.device)
    packed_cu[1:] = lens.cumsum(0).to(torch.int32)
    perm = torch.argsort((~mask).to(torch.int8), stable=True)
    return mask, perm, packed_cu


def _gather(x, perm):
    return x.index_select(0, perm)


def _scatter_rows(dst, src_perm_order, perm, mask):
    """dst[perm[j]] = src[j] for the used rows (mask)."""
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device=perm.device)
    back = src_perm_order.index_select(0, inv)
    m = mask.view(-1, *([1] * (dst.dim() - 1)))
    dst.copy_(torch.where(m, back, dst))


def _sdpa_varlen(q, k, v, cu_q, cu_k, used_q, used_k, causal, scale):
    """Fallback: per-item SDPA (host loop). Returns out rows and lse for used rows."""
    out = torch.zeros_like(q)
    lse = torch.zeros((q.shape[1], q.shape[0]), dtype=torch.float32, device=q.device)
    cq, ck = cu_q.tolist(), cu_k.tolist()
    uq = used_q.tolist() if used_q is not None else [cq[i + 1] - cq[i] for i in range(len(cq) - 1)]
    uk = used_k.tolist() if used_k is not None else [ck[i + 1] - ck[i] for i in range(len(ck) - 1)]
    for i in range(len(cq) - 1):
        if uq[i] == 0 or uk[i] == 0:
            continue
        qi = q[cq[i]:cq[i] + uq[i]].float().transpose(0, 1)
        ki = k[ck[i]:ck[i] + uk[i]].float().transpose(0, 1)
        vi = v[ck[i]:ck[i] + uk[i]].float().transpose(0, 1)
        s = (qi @ ki.transpose(-1, -2)) * scale
        if causal:
            off = uk[i] - uq[i]
            qpos = torch.arange(uq[i], device=q.device)[:, None] + off
            s = s.masked_fill(torch.arange(uk[i], device=q.device)[None, :] > qpos, float("-inf"))
        l = torch.logsumexp(s, -1)
        out[cq[i]:cq[i] + uq[i]] = (torch.softmax(s, -1) @ vi).transpose(0, 1).to(q.dtype)
        lse[:, cq[i]:cq[i] + uq[i]] = l
    return out, lse


def _fwd_impl(q, k, v, out, cu_q, cu_k, used_q, used_k, max_q, max_k, scale, causal):
    T = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if out is None:
        out = torch.zeros_like(q)
    lse_full = torch.zeros((q.shape[1], T), dtype=torch.float32, device=q.device)
    fa2 = _fa2_module()
    if fa2 is None:
        o, lse = _sdpa_varlen(q, k, v, cu_q, cu_k, used_q, used_k, causal, scale)
        mask_q, _, _ = _used_rows(cu_q, used_q, T)
        out.copy_(torch.where(mask_q[:, None, None], o, out))
        return out, torch.where(mask_q[None, :], lse, lse_full)
    mask_q, perm_q, pcu_q = _used_rows(cu_q, used_q, T)
    qg = _gather(q, perm_q)
    if used_k is not None:
        mask_k, perm_k, pcu_k = _used_rows(cu_k, used_k, k.shape[0])
        kg, vg = _gather(k, perm_k), _gather(v, perm_k)
    else:
        kg, vg, pcu_k = k, v, cu_k.to(torch.int32)
    o, lse, _, _ = fa2._flash_attn_varlen_forward(qg, kg, vg, pcu_q, pcu_k, int(max_q), int(max_k), 0.0, scale,
                                                  causal)
    _scatter_rows(out, o, perm_q, mask_q)
    inv = torch.empty_like(perm_q)
    inv[perm_q] = torch.arange(T, device=q.device)
    lse_back = lse[:, :T].index_select(1, inv) if lse.shape[1] >= T else torch.nn.functional.pad(
        lse, (0, T - lse.shape[1])).index_select(1, inv)
    return out, torch.where(mask_q[None, :], lse_back, lse_full)


lib = torch.library.Library("flash_attn_3", "DEF")
lib.define(
    "fwd(Tensor q, Tensor k, Tensor v, Tensor? k_new, Tensor? v_new, Tensor? q_v, Tensor(a!)? out, "
    "Tensor? cu_seqlens_q, Tensor? cu_seqlens_k, Tensor? cu_seqlens_k_new, Tensor? seqused_q, Tensor? seqused_k, "
    "int? max_seqlen_q, int? max_seqlen_k, Tensor? page_table, Tensor? kv_batch_idx, Tensor? leftpad_k, "
    "Tensor? rotary_cos, Tensor? rotary_sin, Tensor? seqlens_rotary, Tensor? q_descale, Tensor? k_descale, "
    "Tensor? v_descale, float? softmax_scale, bool is_causal, int window_size_left, int window_size_right, "
    "int attention_chunk, float softcap, bool is_rotary_interleaved, Tensor? scheduler_metadata, int num_splits, "
    "bool? pack_gqa, int sm_margin) -> (Tensor, Tensor, Tensor, Tensor)")


def _fwd_op(q, k, v, k_new, v_new, q_v, out, cu_seqlens_q, cu_seqlens_k, cu_seqlens_k_new, seqused_q, seqused_k,
            max_seqlen_q, max_seqlen_k, page_table, kv_batch_idx, leftpad_k, rotary_cos, rotary_sin, seqlens_rotary,
            q_descale, k_descale, v_descale, softmax_scale, is_causal, window_size_left, window_size_right,
            attention_chunk, softcap, is_rotary_interleaved, scheduler_metadata, num_splits, pack_gqa, sm_margin):
    o, lse = _fwd_impl(q, k, v, out, cu_seqlens_q, cu_seqlens_k, seqused_q, seqused_k, max_seqlen_q, max_seqlen_k,
                       softmax_scale, is_causal)
    empty = torch.empty(0, device=q.device)
    return o, lse, empty, empty


lib.impl("fwd", _fwd_op, "CUDA")


def _flash_attn_backward(dout, q, k, v, out, softmax_lse, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=None,
                         max_seqlen_k=None, sequed_q=None, sequed_k=None, dq=None, dk=None, dv=None,
                         softmax_scale=None, is_causal=False, **unused):
    T = q.shape[0]
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    fa2 = _fa2_module()
    if fa2 is None:
        return _sdpa_backward(dout, q, k, v, cu_seqlens_q, cu_seqlens_k, sequed_q, sequed_k, dq, dk, dv, scale,
                              is_causal)
    mask_q, perm_q, pcu_q = _used_rows(cu_seqlens_q, sequed_q, T)
    qg, dog, og = _gather(q, perm_q), _gather(dout, perm_q), _gather(out, perm_q)
    inv_lse = softmax_lse.index_select(1, perm_q).contiguous()
    if sequed_k is not None:
        mask_k, perm_k, pcu_k = _used_rows(cu_seqlens_k, sequed_k, k.shape[0])
        kg, vg = _gather(k, perm_k), _gather(v, perm_k)
    else:
        mask_k, perm_k, pcu_k, kg, vg = None, None, cu_seqlens_k.to(torch.int32), k, v
    dqg, dkg, dvg = torch.empty_like(qg), torch.empty_like(kg), torch.empty_like(vg)
    fa2._flash_attn_varlen_backward(dog, qg, kg, vg, og, inv_lse, dqg, dkg, dvg, pcu_q, pcu_k, int(max_seqlen_q),
                                    int(max_seqlen_k), 0.0, scale, is_causal, -1, -1, 0.0, None, False)
    _scatter_rows(dq, dqg, perm_q, mask_q)
    if perm_k is not None:
        _scatter_rows(dk, dkg, perm_k, mask_k)
        _scatter_rows(dv, dvg, perm_k, mask_k)
    else:
        mask_k, _, _ = _used_rows(cu_seqlens_k, None, k.shape[0])
        dk.copy_(torch.where(mask_k[:, None, None], dkg, dk))
        dv.copy_(torch.where(mask_k[:, None, None], dvg, dv))
    return dq, dk, dv


def _sdpa_backward(dout, q, k, v, cu_q, cu_k, used_q, used_k, dq, dk, dv, scale, causal):
    with torch.enable_grad():
        qr, kr, vr = (t.detach().requires_grad_(True) for t in (q, k, v))
        o, _ = _sdpa_varlen(qr, kr, vr, cu_q, cu_k, used_q, used_k, causal, scale)
        o.backward(dout)
    mq, _, _ = _used_rows(cu_q, used_q, q.shape[0])
    mk, _, _ = _used_rows(cu_k, used_k, k.shape[0])
    dq.copy_(torch.where(mq[:, None, None], qr.grad, dq))
    dk.copy_(torch.where(mk[:, None, None], kr.grad, dk))
    dv.copy_(torch.where(mk[:, None, None], vr.grad, dv))
    return dq, dk, dv


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, cache_seqlens=None, causal=False, num_splits=1,
                            **unused):
    """KV-cache attention (inference): append k, v at ``cache_seqlens`` then attend (SDPA)."""
    B, S = q.shape[0], q.shape[1]
    lengths = cache_seqlens if torch.is_tensor(cache_seqlens) else torch.full((B,), int(cache_seqlens or 0),
                                                                              device=q.device)
    lengths = lengths.to(torch.long).view(-1)
    pos = lengths[:, None] + torch.arange(S, device=q.device)[None, :]
    b_idx = torch.arange(B, device=q.device)[:, None].expand(B, S)
    if k is not None:
        k_cache[b_idx, pos] = k
        v_cache[b_idx, pos] = v
    total = lengths + S
    kpos = torch.arange(k_cache.shape[1], device=q.device)
    mask = kpos[None, None, :] < total[:, None, None]
    if causal:
        mask = mask & (kpos[None, None, :] <= pos[:, :, None])
    else:
        mask = mask.expand(B, S, kpos.numel())
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k_cache.transpose(1, 2), v_cache.transpose(1, 2),
                                       attn_mask=mask[:, None])
    return o.transpose(1, 2)
