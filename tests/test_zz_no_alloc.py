"""The allocation-free attention forward (``hrm_attn_fwd_noalloc``), called through its
exported C symbol, must reproduce the regular attention forward.

That entry point serves callers of this library that cannot allocate device memory
themselves (a host runtime that already owns the GPU's memory pool, or a path that cannot
afford cudaMalloc's device synchronisation); its scratch is a static device array in the
library. This file is collected last so that a failure here comes after every other test.
"""
import ctypes

import pytest
import torch

from gpu_utils import assert_close, random_packing

pytestmark = pytest.mark.gpu


def _symbol():
    import hrm_text_b200._C as ext
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.hrm_attn_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_void_p]
    err = lib.hrm_attn_fwd_noalloc_strerror
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


@pytest.mark.parametrize("causal", [False, True])
def test_noalloc_matches_regular_forward(cuda_device, causal):
    from hrm_text_b200.ops.attention import PackedSeq, attention_fwd
    fn, err = _symbol()
    torch.manual_seed(0)
    T, H = 2048, 2
    cu, pl, pos, total = random_packing(T, seed=3)
    cu, pl, pos = cu.to(cuda_device), pl.to(cuda_device), pos.to(cuda_device)
    qkv = torch.randn(T, 4 * H * 128, device=cuda_device).bfloat16()
    ref_out, ref_y, ref_lse = attention_fwd(qkv, H, PackedSeq(pos, cu, pl).schedule(causal), kernel="mma")
    stream = torch.cuda.current_stream(cuda_device)
    for _ in range(2):  # two calls in a row share (and must re-initialise) the static scratch
        out = torch.full_like(ref_out, 7.0)
        y = torch.full_like(ref_y, 7.0)
        lse = torch.full_like(ref_lse, 7.0)
        rc = fn(qkv.data_ptr(), qkv.stride(0), T, H, cu.data_ptr(), cu.numel(), pl.data_ptr(), int(causal),
                out.data_ptr(), y.data_ptr(), out.stride(0), lse.data_ptr(), stream.cuda_stream)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        assert_close(out, ref_out, 1e-3, "O")
        assert_close(y, ref_y, 1e-3, "Y")
        assert_close(lse[:, :total], ref_lse[:, :total], 1e-4, "lse")
        assert out[total:].abs().max().item() == 0.0


def test_noalloc_rejects_oversized_problem(cuda_device):
    fn, err = _symbol()
    T, H = 256, 1
    dummy = torch.zeros(T, 4 * H * 128, dtype=torch.bfloat16, device=cuda_device)
    cu = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = torch.zeros(T, H * 128, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.zeros(H, T, dtype=torch.float32, device=cuda_device)
    rc = fn(dummy.data_ptr(), dummy.stride(0), T, H, cu.data_ptr(), 10 ** 6, cu.data_ptr(), 0, out.data_ptr(),
            out.data_ptr(), out.stride(0), lse.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -1 and b"too large" in err(rc)
