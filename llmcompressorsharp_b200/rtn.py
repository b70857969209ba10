"""Round-to-nearest weight quantisation on the B200.

Mirrors ``RtnConfig`` (src/LLMCompressorSharp.Core/Algorithms/Configs/RtnConfig.cs:17-26) and
``RtnModifier`` (Algorithms/Rtn/RtnModifier.cs:19-123).  One fused pass over each weight
(observer + fake-quant + int packing) for the channel and group strategies.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._device import ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, NotSupportedError
from .gptq import param_shape
from .session import ModifierBase


@dataclass
class RtnConfig:
    num_bits: int = 8
    symmetric: bool = True
    strategy: str = "tensor"
    channel_axis: int = 0
    group_size: int = 128
    targets: list = field(default_factory=list)
    ignore: list = field(default_factory=list)
    type: str = "RTN"

    def to_c(self) -> _lib.QConfig:
        if self.strategy == "token":
            raise NotSupportedError("PerToken strategy applies to activations, not weights.")
        if self.strategy not in _lib.STRATEGY:
            raise ArgumentError(f"Unsupported quantization strategy {self.strategy}.")
        return _lib.QConfig(num_bits=self.num_bits, symmetric=int(self.symmetric), strategy=_lib.STRATEGY[self.strategy],
                            channel_axis=self.channel_axis, group_size=self.group_size, block_size=128)


def rtn_quantize(weight: torch.Tensor, config: RtnConfig, want_codes: bool = True, want_deq: bool = True):
    """Returns (dequantised weight in weight's dtype or None, codes or None, scales, zero_points).
    A 1-D weight is treated as one row."""
    cfg = config.to_c()
    dev = target_device(weight)
    w = to_device(supported_dtype(weight.detach()), dev)
    shape = w.shape
    w2 = w.reshape(1, -1) if w.dim() == 1 else w.reshape(w.shape[0], -1)
    if config.strategy == "channel" and config.channel_axis != 0:
        raise NotSupportedError("RTN on device quantises output channels (axis 0)")
    m, n = w2.shape
    shp = param_shape(config.strategy, m, n, config.group_size)
    scales = torch.empty(shp, dtype=torch.float32, device=dev)
    zps = torch.empty(shp, dtype=torch.int32, device=dev)
    codes = None
    if want_codes and config.num_bits <= 8:
        codes = torch.empty(m, (n + 1) // 2 if config.num_bits <= 4 else n, dtype=torch.uint8, device=dev)
    deq = torch.empty_like(w2) if want_deq else None
    _lib.call("llmc_rtn_quantize", C.c_void_p(ctx(dev)), _lib.ptr(w2), _lib.dtype_code(w2.dtype), C.c_int64(m),
              C.c_int64(n), C.c_int64(n), C.byref(cfg), _lib.ptr(codes), _lib.ptr(scales), _lib.ptr(zps), _lib.ptr(deq))
    if deq is not None:
        deq = deq.reshape(shape)
        if weight.dtype != deq.dtype:
            deq = deq.to(weight.dtype)
        if not weight.is_cuda:
            deq = deq.cpu()
    return deq, codes, scales, zps


class RtnModifier(ModifierBase):
    """RtnModifier.cs:19-123: data-free; OnEnd replaces each targeted weight by its
    fake-quantised value (same dtype) and records the packed codes."""

    def __init__(self, config: RtnConfig):
        if config is None:
            raise ArgumentError("config must not be null")
        super().__init__("RTN", config.targets, config.ignore)
        self.config = config

    def on_initialize(self, state):
        pass

    def on_end_core(self, state):
        for name in self.targeted_names(state):
            w = state.named_weights[name]
            deq, codes, scales, zps = rtn_quantize(w, self.config)
            state.named_weights[name] = deq
            state.compressed[name] = {"codes": codes, "scales": scales, "zero_points": zps,
                                      "num_bits": self.config.num_bits, "symmetric": self.config.symmetric,
                                      "strategy": self.config.strategy, "group_size": self.config.group_size}
