"""Build the in-tree native extensions.

    python setup.py build_ext --inplace

* ``hrm_text_b200._C``    — sm_100a CUDA kernels (csrc/kernels), compiled only for
  ``compute_100a/sm_100a`` with line info. ``HRM_DEBUG_BOUNDS=1`` builds the bounds-checked
  variant (``_C.debug_bounds_build()`` reports which one is loaded).
* ``hrm_text_b200._host`` — host C++ (csrc/host): the multipack LPT allocator.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CUTLASS_INC = os.environ.get("HRM_CUTLASS_INCLUDE", "")

nvcc_flags = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-Xptxas", "-v" if os.environ.get("HRM_PTXAS_VERBOSE") else "-O3",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]

# HRM_DEBUG_BOUNDS=1: bounds-check build (device-side index checks that record the error word)
if os.environ.get("HRM_DEBUG_BOUNDS", "0") == "1":
    nvcc_flags.append("-DHRM_DEBUG_BOUNDS")

cuda_sources = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + ["csrc/kernels/bindings.cpp"]

setup(
    name="hrm_text_b200",
    version="0.1.0",
    packages=["hrm_text_b200"],
    ext_modules=[
        CUDAExtension(
            name="hrm_text_b200._C",
            sources=cuda_sources,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
            libraries=["cuda"],
            library_dirs=["/usr/local/cuda/lib64/stubs"],
        ),
        CppExtension(
            name="hrm_text_b200._host",
            sources=["csrc/host/multipack.cpp"],
            extra_compile_args=["-O3", "-std=c++17"],
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
