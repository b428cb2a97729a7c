"""sm_100a kernel ops.

Every function here takes CUDA tensors and runs this framework's own kernels from the
``hrm_text_b200._C`` extension; there is no alternative backend. CPU tensors are not
accepted (the CPU path of the models is the plain-torch oracle in ``hrm_text_b200.models``).
"""
from .._native import cuda as _cuda  # noqa: F401
