"""Python entry points of the tcgen05 GEMM (csrc/kernels/gemm_tcgen05.cu).

Conventions (row-major tensors, bf16 operands):

* ``linear(x, w)``                 ``y = x @ w.T``            x [M,K], w [N,K]
* ``linear_dgrad(dy, w)``          ``dx = dy @ w``            dy [M,N], w [N,K]
* ``linear_wgrad_(dy, x, grad)``   ``grad += dy.T @ x`` (fp32, stream-K split with atomics)

plus the fused-epilogue variants used by the transformer block and the LM head.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from .._native import cuda

EPI_STORE, EPI_RESIDUAL, EPI_F32ADD, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, EPI_CE = range(7)
EPI_CE_BWD = 8

# Fused collectives (multi-GPU engine): a registered job source hands every GEMM launch the
# copy jobs (weight gather ahead of its first use, gradient push to the owners) that its
# epilogue warps run before their first tile; see hrm_text_b200.parallel.fused.
_job_source = None


def set_job_source(fn) -> None:
    global _job_source
    _job_source = fn


def _check(*tensors: Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("hrm_text_b200.ops.gemm takes CUDA tensors only")
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"GEMM operands must be bf16, got {t.dtype}")


def _gemm(a, a_mn, b, b_mn, M, N, K, epi, out, out2=None, residual=None, aux=None, positions=None, cos=None,
          sin=None, rope_begin=0, rope_end=0, pair_offset=0, labels=None, ce_max=None, ce_sum=None, ce_arg=None,
          ce_tgt=None, stream_k=False, splitk=0):
    jobs = _job_source() if _job_source is not None else None
    cuda().gemm(a, a_mn, b, b_mn, M, N, K, epi, out, out2, residual, aux, positions, cos, sin, rope_begin, rope_end,
                pair_offset, labels, ce_max, ce_sum, ce_arg, ce_tgt, stream_k, splitk, jobs)


def linear(x: Tensor, w: Tensor, out: Optional[Tensor] = None, residual: Optional[Tensor] = None) -> Tensor:
    _check(x, w)
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device) if out is None else out
    _gemm(x, False, w, False, M, N, K, EPI_RESIDUAL if residual is not None else EPI_STORE, out, residual=residual)
    return out


def linear_rope(x: Tensor, w: Tensor, positions: Tensor, cos: Tensor, sin: Tensor, rope_begin: int,
                rope_end: int) -> Tensor:
    """``x @ w.T`` with rotate-half RoPE (head_dim 128) on output columns [rope_begin, rope_end)."""
    _check(x, w)
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _gemm(x, False, w, False, M, N, K, EPI_ROPE, out, positions=positions, cos=cos, sin=sin, rope_begin=rope_begin,
          rope_end=rope_end)
    return out


def linear_swiglu(x: Tensor, w: Tensor) -> tuple[Tensor, Tensor]:
    """For ``w = [gate; up]`` (``[2I, K]``): returns ``(gate|up [M, 2I], silu(gate) * up [M, I])``."""
    _check(x, w)
    M, K = x.shape
    inter = w.shape[0] // 2
    gu = torch.empty((M, 2 * inter), dtype=torch.bfloat16, device=x.device)
    h = torch.empty((M, inter), dtype=torch.bfloat16, device=x.device)
    _gemm(x, False, w, False, M, inter, K, EPI_SWIGLU, gu, out2=h, pair_offset=inter)
    return gu, h


def linear_dgrad(dy: Tensor, w: Tensor, out: Optional[Tensor] = None, residual: Optional[Tensor] = None) -> Tensor:
    _check(dy, w)
    M, N = dy.shape
    K = w.shape[1]
    out = torch.empty((M, K), dtype=torch.bfloat16, device=dy.device) if out is None else out
    _gemm(dy, False, w, True, M, K, N, EPI_RESIDUAL if residual is not None else EPI_STORE, out, residual=residual)
    return out


def linear_dgrad_swiglu(dy: Tensor, w_down: Tensor, gu: Tensor) -> Tensor:
    """``dh = dy @ w_down`` followed by the SwiGLU backward: returns ``d(gate|up) [M, 2I]``."""
    _check(dy, w_down, gu)
    M, N = dy.shape
    inter = w_down.shape[1]
    dgu = torch.empty((M, 2 * inter), dtype=torch.bfloat16, device=dy.device)
    _gemm(dy, False, w_down, True, M, inter, N, EPI_SWIGLU_BWD, dgu, aux=gu, pair_offset=inter)
    return dgu


def linear_wgrad_(dy: Tensor, x: Tensor, grad: Tensor) -> Tensor:
    """``grad += dy.T @ x`` in fp32 (``grad`` is ``[N, K]`` fp32, contiguous)."""
    _check(dy, x)
    assert grad.dtype == torch.float32 and grad.is_contiguous()
    T, N = dy.shape
    K = x.shape[1]
    _gemm(dy, True, x, True, N, K, T, EPI_F32ADD, grad, stream_k=True)
    return grad


def linear_dgrad_accumulate_(dy: Tensor, w: Tensor, acc: Tensor) -> Tensor:
    """``acc += dy @ w`` in fp32 (``acc`` is ``[M, K]`` fp32, contiguous)."""
    _check(dy, w)
    assert acc.dtype == torch.float32 and acc.is_contiguous()
    M, N = dy.shape
    K = w.shape[1]
    _gemm(dy, False, w, True, M, K, N, EPI_F32ADD, acc)
    return acc


def lm_head_ce_stats(x: Tensor, w: Tensor, labels: Tensor):
    """Per-128-column softmax statistics of the logits ``x @ w.T`` (which are not stored):
    ``(row max, sum of exp, argmax)`` per slice ``[2 * n_tiles, M]`` and the label logit ``[M]``."""
    _check(x, w)
    M, K = x.shape
    V = w.shape[0]
    n_tiles = 2 * ((V + 255) // 256)
    pmax = torch.empty((n_tiles, M), dtype=torch.float32, device=x.device)
    psum = torch.empty((n_tiles, M), dtype=torch.float32, device=x.device)
    parg = torch.empty((n_tiles, M), dtype=torch.int32, device=x.device)
    tgt = torch.zeros((M,), dtype=torch.float32, device=x.device)
    no_logits = torch.empty((0,), dtype=torch.bfloat16, device=x.device)
    _gemm(x, False, w, False, M, V, K, EPI_CE, no_logits, labels=labels, ce_max=pmax, ce_sum=psum, ce_arg=parg,
          ce_tgt=tgt)
    return pmax, psum, parg, tgt


def lm_head_ce_dlogits(x: Tensor, w_chunk: Tensor, labels: Tensor, lse: Tensor, grad: Tensor, col0: int,
                       out: Tensor) -> Tensor:
    """``out = (softmax - onehot(labels)) * grad`` for head rows ``[col0, col0 + w_chunk.shape[0])``,
    with the logits recomputed as ``x @ w_chunk.T`` and normalised by the forward's ``lse``."""
    _check(x, w_chunk)
    M, K = x.shape
    N = w_chunk.shape[0]
    _gemm(x, False, w_chunk, False, M, N, K, EPI_CE_BWD, out, labels=labels, ce_max=lse, ce_sum=grad,
          pair_offset=col0)
    return out


# ---------------------------------------------------------------------------------------
# inference: the same layers for any M; decode steps (M <= 128) run the tcgen05 GEMM in
# split-K mode (K spread over all SMs, one fp32 [M, N] slice per K range) and a finishing
# kernel that sums the slices in order and applies the epilogue (csrc/kernels/skinny_gemm.cu)
# ---------------------------------------------------------------------------------------
DECODE_MAX_M = 128
_SM_COUNT: dict = {}


def _decode_gemm(x: Tensor, w: Tensor) -> Tensor:
    M, K = x.shape
    N = w.shape[0]
    dev = x.device
    sms = _SM_COUNT.get(dev)
    if sms is None:
        sms = _SM_COUNT[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    tiles = -(-N // 256)
    split = max(1, min(-(-K // 64), round(2 * sms / tiles)))
    acc = torch.empty((split, M, N), dtype=torch.float32, device=dev)  # every element is written
    _gemm(x, False, w, False, M, N, K, EPI_F32ADD, acc, stream_k=True, splitk=split)
    return acc


def _decode_path(x: Tensor) -> bool:
    return x.shape[0] <= DECODE_MAX_M


def infer_linear(x: Tensor, w: Tensor, residual: Optional[Tensor] = None) -> Tensor:
    """``x @ w.T (+ residual)`` for inference."""
    _check(x, w)
    if not _decode_path(x):
        return linear(x, w, residual=residual)
    acc = _decode_gemm(x, w)
    out = torch.empty((x.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
    cuda().decode_linear_finish(acc, EPI_RESIDUAL if residual is not None else EPI_STORE, out, residual, None, None,
                                None, 0, 0, 0)
    return out


def infer_linear_rope(x: Tensor, w: Tensor, positions: Tensor, cos: Tensor, sin: Tensor, rope_begin: int,
                      rope_end: int) -> Tensor:
    _check(x, w)
    if not _decode_path(x):
        return linear_rope(x, w, positions, cos, sin, rope_begin, rope_end)
    acc = _decode_gemm(x, w)
    out = torch.empty((x.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
    cuda().decode_linear_finish(acc, EPI_ROPE, out, None, positions, cos, sin, rope_begin, rope_end, 0)
    return out


def infer_swiglu(x: Tensor, w: Tensor) -> Tensor:
    """``silu(x @ gate.T) * (x @ up.T)`` for ``w = [gate; up]`` (only ``h`` is produced)."""
    _check(x, w)
    if not _decode_path(x):
        return linear_swiglu(x, w)[1]
    inter = w.shape[0] // 2
    acc = _decode_gemm(x, w)
    h = torch.empty((x.shape[0], inter), dtype=torch.bfloat16, device=x.device)
    cuda().decode_linear_finish(acc, EPI_SWIGLU, h, None, None, None, None, 0, 0, inter)
    return h
