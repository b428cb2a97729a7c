"""Host-side argument checks of the allocation-free attention entry point.

Every case here is rejected before the entry point touches the GPU (no device call, no
launch), so the checks run on a machine without a GPU; the pointers are fake addresses that
are never dereferenced. The GPU behaviour is covered by tests/test_zz_no_alloc.py.
"""
import ctypes

import pytest


def _fn():
    import torch  # noqa: F401  (loads the libraries the extension links against)
    try:
        import hrm_text_b200._C as ext
    except ImportError:
        pytest.skip("native extension not built")
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.hrm_attn_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_void_p]
    return fn


MAX_TILES = ((1 << 20) // 4 - 8 - 4) // 8
A = 1 << 20  # a fake, 256-byte aligned "device" address


def _args(**kw):
    H, T = 2, 1024
    a = dict(qkv=A, ld_qkv=4 * H * 128, T=T, H=H, cu=A + 4096, n_cu=5, pl=A + 8192, causal=0, out=A + 16384,
             y=A + 32768, ld_out=H * 128, lse=A + 65536, stream=None)
    a.update(kw)
    return [a[k] for k in ("qkv", "ld_qkv", "T", "H", "cu", "n_cu", "pl", "causal", "out", "y", "ld_out", "lse",
                           "stream")]


@pytest.mark.parametrize("bad", [
    dict(qkv=0), dict(out=0), dict(y=0), dict(lse=0), dict(cu=0), dict(pl=0),
    dict(qkv=A + 8), dict(out=A + 16384 + 2), dict(y=A + 32768 + 4), dict(lse=A + 65536 + 2), dict(cu=A + 4097),
    dict(pl=A + 8194), dict(ld_qkv=4 * 2 * 128 - 8), dict(ld_qkv=4 * 2 * 128 + 4), dict(ld_out=2 * 128 + 4),
    dict(ld_out=128), dict(T=0), dict(H=0), dict(n_cu=0),
])
def test_rejected_before_any_device_call(bad):
    assert _fn()(*_args(**bad)) == -2


def test_tile_limit_checked_on_the_host():
    fn = _fn()
    T = 1024
    assert fn(*_args(T=T, n_cu=MAX_TILES - T // 128 + 1)) == -1
    assert fn(*_args(T=T, n_cu=10 ** 6)) == -1
