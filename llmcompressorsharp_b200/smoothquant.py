"""SmoothQuant on the B200.

Mirrors ``SmoothQuantConfig`` / ``SmoothQuantMapping`` (src/LLMCompressorSharp.Core/Algorithms/
Configs/SmoothQuantConfig.cs:14-34, SmoothQuantMapping.cs:14) and ``SmoothQuantModifier``
(Algorithms/SmoothQuant/SmoothQuantModifier.cs:15-183).  The running activation absmax is
a device vector; the smoothing scale, division and multiplication run in one kernel.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._device import ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, ArgumentOutOfRangeError, InvalidOperationError
from .session import ModifierBase


@dataclass(frozen=True)
class SmoothQuantMapping:
    smooth_weight: str
    balance_weight: str
    activation_key: str


@dataclass
class SmoothQuantConfig:
    smoothing_strength: float = 0.5
    mappings: list = field(default_factory=list)
    targets: list = field(default_factory=list)
    ignore: list = field(default_factory=list)
    type: str = "SmoothQuant"


def act_absmax(x: torch.Tensor, running: torch.Tensor | None = None) -> torch.Tensor:
    """|x|.amax over all dims but the last, folded into ``running`` (fp32 device vector)."""
    dev = running.device if running is not None else target_device(x)
    xd = to_device(supported_dtype(x.detach()), dev)
    cols = xd.shape[-1]
    x2 = xd.reshape(-1, cols)
    out = running if running is not None else torch.empty(cols, dtype=torch.float32, device=dev)
    _lib.call("llmc_act_absmax", C.c_void_p(ctx(dev)), _lib.ptr(x2), _lib.dtype_code(x2.dtype), C.c_int64(x2.shape[0]),
              C.c_int64(cols), C.c_int64(cols), _lib.ptr(out), C.c_int32(1 if running is not None else 0))
    return out


def smooth_apply(smooth_w: torch.Tensor, balance_w: torch.Tensor, act_max: torch.Tensor, alpha: float):
    """ApplyMapping (:117-182) on device copies; returns (new_smooth, new_balance, s)."""
    dev = target_device(smooth_w, balance_w, act_max)
    sw = to_device(supported_dtype(smooth_w.detach()), dev).clone()
    bw = to_device(supported_dtype(balance_w.detach()), dev).clone()
    am = to_device(act_max.detach(), dev, torch.float32)
    s = torch.empty(sw.shape[0], dtype=torch.float32, device=dev)
    _lib.call("llmc_smooth_apply", C.c_void_p(ctx(dev)), _lib.ptr(am), _lib.ptr(sw), _lib.dtype_code(sw.dtype),
              _lib.ptr(bw), _lib.dtype_code(bw.dtype), C.c_int64(bw.shape[0]), C.c_int64(bw.shape[1]),
              C.c_float(alpha), _lib.ptr(s))
    if not smooth_w.is_cuda:
        sw = sw.cpu()
    if not balance_w.is_cuda:
        bw = bw.cpu()
    return sw, bw, s


class SmoothQuantModifier(ModifierBase):
    def __init__(self, config: SmoothQuantConfig):
        if config is None:
            raise ArgumentError("config must not be null")
        if not (0.0 <= config.smoothing_strength <= 1.0):
            raise ArgumentOutOfRangeError("SmoothingStrength (alpha) must be in [0, 1].")
        super().__init__("SmoothQuant", config.targets, config.ignore)
        self.config = config
        self._running: dict[str, torch.Tensor] = {}

    def on_initialize(self, state):
        self._running.clear()

    def on_batch_core(self, state):  # :44-60
        if state.layer_activations is None:
            return
        for mp in self.config.mappings:
            x = state.layer_activations.get(mp.activation_key)
            if x is not None:
                self._update(mp.activation_key, x)

    def _update(self, key, x):
        cur = self._running.get(key)
        if cur is not None and cur.shape[0] != x.shape[-1]:
            raise InvalidOperationError(
                f"SmoothQuant: activation feature dim changed for '{key}': expected {cur.shape[0]}, got {x.shape[-1]}.")
        self._running[key] = act_absmax(x, cur)

    def on_end_core(self, state):
        for mp in self.config.mappings:
            self._apply(state, mp)

    def _apply(self, state, mp: SmoothQuantMapping):  # :117-182
        x = state.layer_activations.get(mp.activation_key) if state.layer_activations is not None else None
        if x is None:
            if mp.activation_key not in self._running:
                raise InvalidOperationError(
                    f"SmoothQuant: no activation collected for '{mp.activation_key}'. "
                    "Populate CompressionState.LayerActivations.")
        elif mp.activation_key not in self._running:
            self._update(mp.activation_key, x)
        amax = self._running[mp.activation_key]
        sw = state.named_weights[mp.smooth_weight]
        if sw.dim() != 1:
            raise InvalidOperationError(
                f"SmoothQuant: smooth weight '{mp.smooth_weight}' must be 1-D (got rank {sw.dim()}).")
        bw = state.named_weights[mp.balance_weight]
        if bw.dim() != 2:
            raise InvalidOperationError(
                f"SmoothQuant: balance weight '{mp.balance_weight}' must be 2-D (got rank {bw.dim()}).")
        hidden = sw.shape[0]
        if amax.shape[0] != hidden:
            raise InvalidOperationError(
                f"SmoothQuant: activation hidden dim {amax.shape[0]} does not match smooth weight {hidden}.")
        if bw.shape[1] != hidden:
            raise InvalidOperationError(
                f"SmoothQuant: balance weight last dim {bw.shape[1]} does not match hidden {hidden}.")
        new_s, new_b, _ = smooth_apply(sw, bw, amax, self.config.smoothing_strength)
        state.named_weights[mp.smooth_weight] = new_s
        state.named_weights[mp.balance_weight] = new_b
