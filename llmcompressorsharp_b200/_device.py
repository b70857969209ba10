"""Device placement helpers: every compute call runs on a CUDA device through the C ABI.

Host (CPU) tensors are accepted the way the reference accepts them and are staged to the
current CUDA device with a pinned, asynchronous copy; results then return to the host.
"""

from __future__ import annotations

import torch

from . import _lib


class DeviceView:
    """Zero-copy torch view of a device buffer the library owns (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3, "strides": None,
        }


def target_device(*tensors) -> torch.device:
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("llmcompressorsharp_b200 needs a CUDA device (B200); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def to_device(t: torch.Tensor, device: torch.device, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Contiguous copy/view of t on device (pinned async H2D for host tensors)."""
    if dtype is not None and t.dtype != dtype and t.device.type == "cpu":
        t = t.to(dtype)
    if t.device != device:
        if t.device.type == "cpu":
            t = t.contiguous()
            if not t.is_pinned():
                t = t.pin_memory()
            t = t.to(device, non_blocking=True)
        else:
            t = t.to(device)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def supported_dtype(t: torch.Tensor) -> torch.Tensor:
    if t.dtype in (torch.float32, torch.bfloat16, torch.float16):
        return t
    return t.to(torch.float32)


def ctx(device: torch.device) -> int:
    return _lib.ctx_for(device.index if device.index is not None else torch.cuda.current_device())
