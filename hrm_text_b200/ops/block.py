"""Fused transformer layer on sm_100a kernels (one autograd node per layer).

Forward of a pre-norm layer (reference models/transformer.py:90-92, models/layers.py:129-168):

    s   = x (+ injection)                      fused into the first RMSNorm
    xn  = rmsnorm(s)
    g|q|k|v = xn @ Wgqkv^T, RoPE on q, k       GEMM with RoPE epilogue
    O, Y = attention(q, k, v), Y = sigmoid(g) * O   flash attention, gate in the epilogue
    x1  = s + Y @ Wo^T                         GEMM with residual epilogue
    xn2 = rmsnorm(x1)
    gu, h = xn2 @ Wgu^T, h = silu(gate) * up   GEMM with SwiGLU epilogue
    x2  = x1 + h @ Wd^T                        GEMM with residual epilogue

The backward is written out by hand (no autograd inside): dgrad GEMMs with fused SwiGLU /
residual epilogues, fp32 weight-gradient GEMMs accumulating straight into each weight's
``main_grad`` buffer (so the gradients of the 2-3 recurrent calls that reuse a layer add
up in fp32 without extra passes), and the flash-attention backward with the gate and RoPE
backward fused. Weight tensors are the bf16 compute copies; when a weight has no
``main_grad`` the node returns an ordinary gradient instead.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .._native import cuda
from ..parallel.fused import before_use
from ..utils.trace import nvtx
from . import gemm as G
from .attention import PackedSeq, attention_bwd, attention_fwd, rope_half_tables


def rmsnorm(x: Tensor, eps: float, injection: Tensor | None = None):
    """Returns ``(y, rstd, s)``; ``s = bf16(x + injection)`` when an injection is given (else ``x``)."""
    T, H = (injection.shape if injection is not None else x.shape)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=(injection if injection is not None else x).device)
    rstd = torch.empty((T,), dtype=torch.float32, device=y.device)
    if injection is not None:
        s = torch.empty_like(y)
        cuda().rmsnorm_fwd(x, injection, s, y, rstd, T, eps)
    else:
        cuda().rmsnorm_fwd(x, None, None, y, rstd, T, eps)
        s = x
    return y, rstd, s


def rmsnorm_bwd(dy: Tensor, s: Tensor, rstd: Tensor, dres: Tensor | None = None) -> Tensor:
    dx = torch.empty_like(dy)
    cuda().rmsnorm_bwd(dy, s, rstd, dres, dx, dy.shape[0])
    return dx


def _wgrad(dy: Tensor, x: Tensor, w: Tensor, grads: list, idx: int) -> None:
    f2 = getattr(w, "_f2", None)
    if f2 is not None:
        w._f2_pending -= 1
        if f2.enabled and w._f2_pending == 0:  # last contribution of this step
            G.linear_wgrad_(dy, x, w.main_grad)
            f2.owner.queue_push(f2)  # the next GEMM pushes the finished rows to their owners
            return
    main = getattr(w, "main_grad", None)
    if main is not None:
        G.linear_wgrad_(dy, x, main)
    else:
        g = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        G.linear_wgrad_(dy, x, g)
        grads[idx] = g.to(w.dtype)


class FusedPreNormBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, injection, w_gqkv, w_o, w_gu, w_d, packed: PackedSeq, rope, num_heads: int, eps: float,
                causal: bool, train: bool):
        cos, sin = rope
        hidden = w_o.shape[0]
        with nvtx("rmsnorm.fwd"):
            xn, r1, s = rmsnorm(x, eps, injection)
        sched = packed.schedule(causal)
        # multi-GPU fused path: before_use makes sure a sharded weight's resident copy is gathered
        # (normally by a copy job inside an earlier GEMM of the step) before its first GEMM
        with nvtx("gemm.gqkv_rope"):
            before_use(w_gqkv)
            gqkv = G.linear_rope(xn, w_gqkv, packed.position_ids, cos, sin, hidden, 3 * hidden)
        with nvtx("attention.fwd"):
            o, y, lse = attention_fwd(gqkv, num_heads, sched)
        with nvtx("gemm.o_residual"):
            before_use(w_o)
            x1 = G.linear(y, w_o, residual=s)
        with nvtx("rmsnorm.fwd"):
            xn2, r2, _ = rmsnorm(x1, eps)
        with nvtx("gemm.gate_up_swiglu"):
            before_use(w_gu)
            gu, h = G.linear_swiglu(xn2, w_gu)
        with nvtx("gemm.down_residual"):
            before_use(w_d)
            x2 = G.linear(h, w_d, residual=x1)
        if train:
            for w in (w_gqkv, w_o, w_gu, w_d):
                if getattr(w, "_f2", None) is not None:
                    w._f2_pending += 1
            ctx.weights = (w_gqkv, w_o, w_gu, w_d)
            ctx.save_for_backward(s, r1, xn, gqkv, o, lse, y, x1, r2, xn2, gu, h, w_gqkv, w_o, w_gu, w_d, cos, sin)
            ctx.packed, ctx.num_heads, ctx.causal = packed, num_heads, causal
            ctx.has_injection = injection is not None
        return x2

    @staticmethod
    def backward(ctx, dx2):
        (s, r1, xn, gqkv, o, lse, y, x1, r2, xn2, gu, h, _, _, _, _, cos, sin) = ctx.saved_tensors
        w_gqkv, w_o, w_gu, w_d = ctx.weights  # the parameter objects (carry main_grad / F2 metadata)
        packed = ctx.packed
        dx2 = dx2.contiguous()
        grads = [None] * 4
        # MLP
        with nvtx("gemm.down_dgrad_swiglu"):
            dgu = G.linear_dgrad_swiglu(dx2, w_d, gu)
        with nvtx("gemm.wgrad"):
            _wgrad(dx2, h, w_d, grads, 3)
        with nvtx("gemm.dgrad"):
            dxn2 = G.linear_dgrad(dgu, w_gu)
        with nvtx("gemm.wgrad"):
            _wgrad(dgu, xn2, w_gu, grads, 2)
        with nvtx("rmsnorm.bwd"):
            dx1 = rmsnorm_bwd(dxn2, x1, r2, dres=dx2)
        # attention
        with nvtx("gemm.dgrad"):
            dy = G.linear_dgrad(dx1, w_o)
        with nvtx("gemm.wgrad"):
            _wgrad(dx1, y, w_o, grads, 1)
        with nvtx("attention.bwd"):
            dgqkv = attention_bwd(gqkv, ctx.num_heads, packed.schedule(ctx.causal), o, lse, dy,
                                  packed.position_ids, cos, sin)
        with nvtx("gemm.dgrad"):
            dxn = G.linear_dgrad(dgqkv, w_gqkv)
        with nvtx("gemm.wgrad"):
            _wgrad(dgqkv, xn, w_gqkv, grads, 0)
        with nvtx("rmsnorm.bwd"):
            ds = rmsnorm_bwd(dxn, s, r1, dres=dx1)
        d_inj = ds if ctx.has_injection else None
        return (ds, d_inj, grads[0], grads[1], grads[2], grads[3], None, None, None, None, None, None)


class FinalNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps: float):
        y, rstd, _ = rmsnorm(x, eps)
        ctx.save_for_backward(x, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, rstd = ctx.saved_tensors
        return rmsnorm_bwd(dy.contiguous(), x, rstd), None


def stack_forward(stack, x: Tensor, injection: Tensor | None, seq_info: dict) -> Tensor:
    """Run ``hrm_text_b200.models.transformer.Transformer`` on the fused CUDA path."""
    cfg = stack.config
    if cfg.norm_type != "pre":
        raise NotImplementedError("the fused CUDA block implements pre-norm layers (all shipped sizes)")
    if cfg.head_dim != 128:
        raise NotImplementedError("the fused CUDA block is specialised for head_dim 128")
    if not hasattr(stack, "rotary_emb"):
        raise NotImplementedError("the fused CUDA block applies RoPE (pos_emb_type 'rope')")
    packed = PackedSeq.from_seq_info(seq_info)
    rope = rope_half_tables(stack.rotary_emb)
    causal = cfg.attn_type == "causal"
    train = torch.is_grad_enabled()
    if injection is not None and x.dim() == 1:  # broadcast initial state (zL_init)
        x = x.to(injection.dtype).expand_as(injection)
    if x.dim() == 2 and x.stride(0) == 0:
        x = x.contiguous()
    for i, layer in enumerate(stack.layers):
        a, m = layer.attn, layer.mlp
        x = FusedPreNormBlock.apply(x, injection if i == 0 else None, a.gqkv_proj.weight, a.o_proj.weight,
                                    m.gate_up_proj.weight, m.down_proj.weight, packed, rope, a.num_heads,
                                    cfg.norm_eps, causal, train)
    return FinalNorm.apply(x, cfg.norm_eps)


def stack_forward_cached(stack, x: Tensor, injection: Tensor | None, cache: list, cache_lengths,
                         position_ids: Tensor) -> Tensor | None:
    """Inference forward of a pre-norm ``Transformer`` stack against static KV caches, on the
    framework's kernels (reference models/layers.py:129-168 with ``flash_attn_with_kvcache``,
    simple_inference_engine.py:105-112).

    Two shapes of call run here; anything else returns ``None`` (the caller then uses the
    torch reference path):

    * decode: ``x [B, 1, h]``, ``cache_lengths`` a ``[B]`` tensor. Per layer: RMSNorm kernel,
      gqkv projection with RoPE at positions ``cache_lengths`` (tcgen05 GEMM in split-K mode
      plus the epilogue kernel of skinny_gemm.cu), one decode
      attention call that appends the step's keys / values to the caches, attends over
      ``[0, cache_lengths + 1)`` and applies the sigmoid gate, then the o_proj GEMM with the
      residual epilogue, RMSNorm, the gate/up GEMM with the SwiGLU epilogue and the down GEMM
      with the residual epilogue;
    * prefill of one prompt into an empty cache: ``x [1, L, h]``, ``cache_lengths == 0``. The
      same GEMMs, the prompt's keys / values copied into the caches, and the tcgen05 PrefixLM
      forward over the prompt (bidirectional; causal for a causal stack).

    Every launch is a device-side operation on static shapes, so a decode step can be captured
    in a CUDA graph.
    """
    cfg = stack.config
    if cfg.norm_type != "pre" or cfg.head_dim != 128 or not hasattr(stack, "rotary_emb"):
        return None
    ref = injection if injection is not None else x
    if ref.dim() != 3:
        return None
    B, S, hidden = ref.shape
    decode = S == 1 and isinstance(cache_lengths, Tensor) and cache_lengths.numel() == B
    prefill = B == 1 and isinstance(cache_lengths, int) and cache_lengths == 0
    if not (decode or prefill):
        return None
    cos, sin = rope_half_tables(stack.rotary_emb)
    causal = cfg.attn_type == "causal"
    T = B * S
    if x.dim() == 1:  # broadcast initial state (zL_init)
        x = x.to(ref.dtype).expand(T, hidden).contiguous()
    else:
        x = x.reshape(T, hidden)
    inj = injection.reshape(T, hidden).contiguous() if injection is not None else None
    positions = position_ids.reshape(-1).to(torch.int32).contiguous()
    if decode:
        lengths = cache_lengths.to(device=x.device, dtype=torch.int32).contiguous()
    else:
        cu = torch.tensor([0, S], dtype=torch.int32, device=x.device)
        pl = torch.tensor([0 if causal else S], dtype=torch.int32, device=x.device)
        packed = PackedSeq(positions, cu, pl)
        sched = packed.schedule(causal)
    for i, layer in enumerate(stack.layers):
        a, m = layer.attn, layer.mlp
        H = a.num_heads
        c = cache[i]
        xn, _, s = rmsnorm(x, cfg.norm_eps, inj if i == 0 else None)
        gqkv = G.infer_linear_rope(xn, a.gqkv_proj.weight, positions, cos, sin, hidden, 3 * hidden)
        if decode:
            y = cuda().decode_attention_gqkv(gqkv, H, c.keys, c.values, lengths)
        else:
            heads = gqkv.view(S, 4, H, 128)
            c.keys[0, :S].copy_(heads[:, 2])
            c.values[0, :S].copy_(heads[:, 3])
            _, y, _ = attention_fwd(gqkv, H, sched)
        x1 = G.infer_linear(y, a.o_proj.weight, residual=s)
        xn2, _, _ = rmsnorm(x1, cfg.norm_eps)
        h = G.infer_swiglu(xn2, m.gate_up_proj.weight)
        x = G.infer_linear(h, m.down_proj.weight, residual=x1)
    out, _, _ = rmsnorm(x, cfg.norm_eps)
    return out.view(B, S, hidden)
