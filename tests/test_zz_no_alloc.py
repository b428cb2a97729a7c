"""The allocation-free attention forward (``hrm_attn_fwd_noalloc``), called through its
exported C symbol, must reproduce the regular (tcgen05) attention forward.

That entry point serves callers of this library that cannot allocate device memory
themselves: a host runtime that already owns the GPU's memory pool, or a path that cannot
afford cudaMalloc's implicit device synchronisation. Its scratch (work schedule, counters,
error word) is a static device array inside the library. This file is collected last so that
a failure here comes after every other test has run.
"""
import ctypes

import pytest
import torch

from gpu_utils import assert_close, random_packing

pytestmark = pytest.mark.gpu

SCRATCH_INTS = (1 << 20) // 4
MAX_TILES = (SCRATCH_INTS - 8 - 4) // 8  # HRM_ATTN_NOALLOC_MAX_TILES


def _lib():
    import hrm_text_b200._C as ext
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.hrm_attn_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_void_p]
    lib.hrm_attn_fwd_noalloc_strerror.restype = ctypes.c_char_p
    lib.hrm_attn_fwd_noalloc_strerror.argtypes = [ctypes.c_int]
    lib.hrm_attn_fwd_noalloc_status.restype = ctypes.c_int
    lib.hrm_attn_fwd_noalloc_status.argtypes = [ctypes.c_void_p]
    return lib


def _status(lib):
    word = (ctypes.c_int * 4)()
    assert lib.hrm_attn_fwd_noalloc_status(word) == 0
    return list(word)


def _call(lib, qkv, T, H, cu, n_cu, pl, causal, out, y, lse, stream=None):
    stream = torch.cuda.current_stream() if stream is None else stream
    return lib.hrm_attn_fwd_noalloc(qkv.data_ptr(), qkv.stride(0), T, H, cu.data_ptr(), n_cu, pl.data_ptr(),
                                    int(causal), out.data_ptr(), y.data_ptr(), out.stride(0), lse.data_ptr(),
                                    stream.cuda_stream)


@pytest.mark.parametrize("causal", [False, True])
def test_noalloc_matches_regular_forward(cuda_device, causal):
    from hrm_text_b200.ops.attention import PackedSeq, attention_fwd
    lib = _lib()
    torch.manual_seed(0)
    T, H = 2048, 2
    cu, pl, pos, total = random_packing(T, seed=3)
    cu, pl, pos = cu.to(cuda_device), pl.to(cuda_device), pos.to(cuda_device)
    qkv = torch.randn(T, 4 * H * 128, device=cuda_device).bfloat16()
    ref_out, ref_y, ref_lse = attention_fwd(qkv, H, PackedSeq(pos, cu, pl).schedule(causal), kernel="tcgen05")
    for _ in range(2):  # two calls in a row share (and must re-initialise) the static scratch
        out = torch.full_like(ref_out, 7.0)
        y = torch.full_like(ref_y, 7.0)
        lse = torch.full_like(ref_lse, 7.0)
        rc = _call(lib, qkv, T, H, cu, cu.numel(), pl, causal, out, y, lse)
        assert rc == 0, lib.hrm_attn_fwd_noalloc_strerror(rc).decode()
        torch.cuda.synchronize()
        assert _status(lib)[0] == 0
        assert_close(out, ref_out, 1e-3, "O")
        assert_close(y, ref_y, 1e-3, "Y")
        assert_close(lse[:, :total], ref_lse[:, :total], 1e-4, "lse")
        assert out[total:].abs().max().item() == 0.0 and y[total:].abs().max().item() == 0.0


def test_noalloc_tile_limit_is_exact(cuda_device):
    """ceil(T/128) + n_cu == MAX_TILES is accepted (zero-padded cu_seqlens), one more is rejected."""
    from hrm_text_b200.ops.attention import PackedSeq, attention_fwd
    lib = _lib()
    torch.manual_seed(1)
    T, H = 256, 1
    n_cu = MAX_TILES - T // 128
    cu = torch.zeros(n_cu + 1, dtype=torch.int32)
    cu[1:4] = torch.tensor([100, 180, 250], dtype=torch.int32)
    pl = torch.zeros(n_cu + 1, dtype=torch.int32)
    pl[:3] = torch.tensor([40, 0, 70], dtype=torch.int32)
    pos = torch.cat([torch.arange(100), torch.arange(80), torch.arange(70), torch.zeros(6, dtype=torch.long)])
    cu, pl, pos = cu.to(cuda_device), pl.to(cuda_device), pos.int().to(cuda_device)
    qkv = torch.randn(T, 4 * H * 128, device=cuda_device).bfloat16()
    ref_out, _, _ = attention_fwd(qkv, H, PackedSeq(pos, cu[:5], pl[:4]).schedule(False), kernel="tcgen05")
    out = torch.full_like(ref_out, 7.0)
    y, lse = torch.empty_like(out), torch.empty(H, T, device=cuda_device)
    rc = _call(lib, qkv, T, H, cu, n_cu, pl, False, out, y, lse)
    assert rc == 0, lib.hrm_attn_fwd_noalloc_strerror(rc).decode()
    torch.cuda.synchronize()
    assert _status(lib)[0] == 0
    assert_close(out, ref_out, 1e-3, "O at the tile limit")
    rc = _call(lib, qkv, T, H, cu, n_cu + 1, pl, False, out, y, lse)
    assert rc == -1 and b"too large" in lib.hrm_attn_fwd_noalloc_strerror(rc)


def test_noalloc_rejects_bad_arguments(cuda_device):
    lib = _lib()
    T, H = 256, 1
    qkv = torch.zeros(T + 1, 4 * H * 128, dtype=torch.bfloat16, device=cuda_device)
    cu = torch.tensor([0, T, 0], dtype=torch.int32, device=cuda_device)
    pl = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    out = torch.zeros(T + 1, H * 128, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.zeros(H, T + 1, dtype=torch.float32, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    base = [qkv.data_ptr(), qkv.stride(0), T, H, cu.data_ptr(), 3, pl.data_ptr(), 0, out.data_ptr(), out.data_ptr(),
            out.stride(0), lse.data_ptr(), stream]
    assert lib.hrm_attn_fwd_noalloc(*base) == 0
    torch.cuda.synchronize()
    bad = {0: qkv.data_ptr() + 8, 8: out.data_ptr() + 2, 9: out.data_ptr() + 4, 11: lse.data_ptr() + 2,
           4: cu.data_ptr() + 1, 1: 4 * H * 128 - 8, 10: H * 128 + 4, 3: 0, 2: 0}
    for pos, value in bad.items():
        args = list(base)
        args[pos] = value
        rc = lib.hrm_attn_fwd_noalloc(*args)
        assert rc == -2, (pos, rc)
    args = list(base)
    args[5] = 10 ** 6
    assert lib.hrm_attn_fwd_noalloc(*args) == -1


def test_noalloc_rejects_packing_past_T(cuda_device):
    """A last boundary beyond T is rejected on the device: every output row is zero and the
    error word says so; nothing outside the T rows is touched."""
    lib = _lib()
    T, H = 384, 1
    qkv = torch.randn(T, 4 * H * 128, device=cuda_device).bfloat16()
    guard = torch.full((T + 64, H * 128), 3.0, dtype=torch.bfloat16, device=cuda_device)
    out = guard[:T]
    y = torch.full_like(out, 5.0)
    lse = torch.full((H, T), 9.0, device=cuda_device)
    cu = torch.tensor([0, 200, T + 50, 0], dtype=torch.int32, device=cuda_device)
    pl = torch.tensor([10, 20, 0], dtype=torch.int32, device=cuda_device)
    rc = _call(lib, qkv, T, H, cu, 4, pl, False, out, y, lse)
    assert rc == 0
    torch.cuda.synchronize()
    assert _status(lib)[0] == 4
    assert out.abs().max().item() == 0.0 and y.abs().max().item() == 0.0 and lse.abs().max().item() == 0.0
    assert (guard[T:] == 3.0).all().item()
    # the next valid call clears the error word
    cu = torch.tensor([0, 200, T, 0], dtype=torch.int32, device=cuda_device)
    assert _call(lib, qkv, T, H, cu, 4, pl, False, out, y, lse) == 0
    torch.cuda.synchronize()
    assert _status(lib)[0] == 0
