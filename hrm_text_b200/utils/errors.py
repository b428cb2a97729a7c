"""Host side of the device error word.

Every bounded spin-wait in the kernels records ``(code, site, block, thread)`` in a
per-device int32[4] word instead of hanging; ``check_device_errors`` reads it (a device
sync) and raises ``DeviceWaitTimeout`` if a kernel gave up waiting.
"""
from __future__ import annotations

import torch

ERROR_NAMES = {1: "GEMM pipeline wait timed out", 2: "attention wait timed out", 3: "peer flag wait timed out",
               4: "bounds check failed"}


class DeviceWaitTimeout(RuntimeError):
    pass


def error_word() -> torch.Tensor:
    from .._native import cuda
    return cuda().device_error_word()


def check_device_errors(reset: bool = True) -> None:
    word = error_word()
    host = word.cpu().tolist()
    if host[0] != 0:
        if reset:
            word.zero_()
        raise DeviceWaitTimeout(f"{ERROR_NAMES.get(host[0], 'error')} (code {host[0]}, site {host[1]}, "
                                f"block {host[2]}, thread {host[3]})")
