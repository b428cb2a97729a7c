"""Loading of the in-tree native extensions.

* ``_host`` — host C++ (multipack LPT allocator). Built with g++ + pybind11 on first use if
  the shared object is missing (a few seconds), so CPU-only checkouts work.
* ``_C`` — the sm_100a CUDA kernels (``csrc/kernels``), built by ``setup.py build_ext
  --inplace`` (``__graft_entry__.build``). There is no fallback: on a machine with a GPU,
  every CUDA op raises if ``_C`` cannot be imported.
"""
from __future__ import annotations

import importlib
import os
import subprocess
import sys
import sysconfig

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_REPO_DIR = os.path.dirname(_PKG_DIR)

_host_mod = None
_cuda_mod = None


def build_host(verbose: bool = False) -> str:
    """Compile ``csrc/host/*.cpp`` into ``hrm_text_b200/_host<ext-suffix>``."""
    import pybind11

    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    out = os.path.join(_PKG_DIR, f"_host{suffix}")
    src = os.path.join(_REPO_DIR, "csrc", "host", "multipack.cpp")
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC", "-Wall",
           f"-I{sysconfig.get_paths()['include']}", f"-I{pybind11.get_include()}", src, "-o", out]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    return out


def host():
    global _host_mod
    if _host_mod is None:
        try:
            _host_mod = importlib.import_module("hrm_text_b200._host")
        except ImportError:
            build_host()
            importlib.invalidate_caches()
            _host_mod = importlib.import_module("hrm_text_b200._host")
    return _host_mod


class NativeExtensionMissing(RuntimeError):
    pass


def cuda():
    """The CUDA kernel extension; raises ``NativeExtensionMissing`` if it is not built."""
    global _cuda_mod
    if _cuda_mod is None:
        try:
            _cuda_mod = importlib.import_module("hrm_text_b200._C")
        except ImportError as exc:  # pragma: no cover - depends on the build
            raise NativeExtensionMissing(
                "hrm_text_b200._C is not built. Run `python setup.py build_ext --inplace` "
                f"(or __graft_entry__.build()) in {_REPO_DIR}. Import error: {exc}") from exc
    return _cuda_mod


def cuda_available() -> bool:
    try:
        cuda()
        return True
    except NativeExtensionMissing:
        return False


if __name__ == "__main__":  # pragma: no cover
    print(build_host(verbose=True), file=sys.stderr)
