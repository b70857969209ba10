"""AWQ scale search on the B200 (the reference sketches AWQ in
docs/llmcompressorsharp/algorithm-mapping.md:214-249: a grid of alpha = k/nGrid, s =
actMax^alpha / wMax^(1-alpha), keep the s minimising the fake-quant MSE, then apply it as
SmoothQuant applies its scale)."""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._device import ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, InvalidOperationError
from .rtn import RtnConfig
from .session import ModifierBase
from .smoothquant import SmoothQuantMapping, act_absmax


@dataclass
class AWQConfig:
    num_bits: int = 4
    symmetric: bool = False
    strategy: str = "group"
    group_size: int = 128
    n_grid: int = 20
    mappings: list = field(default_factory=list)
    targets: list = field(default_factory=list)
    ignore: list = field(default_factory=list)
    type: str = "AWQ"

    def quant(self) -> RtnConfig:
        return RtnConfig(num_bits=self.num_bits, symmetric=self.symmetric, strategy=self.strategy,
                         group_size=self.group_size)


def awq_search(weight: torch.Tensor, act_max: torch.Tensor, n_grid: int, quant: RtnConfig):
    """Returns (best scale fp32 [n], best k (1-based), mse per grid point fp64 [n_grid])."""
    dev = target_device(weight, act_max)
    w = to_device(supported_dtype(weight.detach()), dev)
    a = to_device(act_max.detach(), dev, torch.float32)
    m, n = w.shape
    best = torch.empty(n, dtype=torch.float32, device=dev)
    mse = torch.empty(n_grid, dtype=torch.float64, device=dev)
    k = C.c_int32()
    cfg = quant.to_c()
    _lib.call("llmc_awq_search", C.c_void_p(ctx(dev)), _lib.ptr(w), _lib.dtype_code(w.dtype), C.c_int64(m),
              C.c_int64(n), C.c_int64(n), _lib.ptr(a), C.c_int32(n_grid), C.byref(cfg), _lib.ptr(best), _lib.ptr(mse),
              C.byref(k))
    return best, int(k.value), mse


def scale_apply(smooth_w: torch.Tensor | None, balance_w: torch.Tensor, s: torch.Tensor):
    dev = target_device(balance_w, s)
    bw = to_device(supported_dtype(balance_w.detach()), dev).clone()
    sw = to_device(supported_dtype(smooth_w.detach()), dev).clone() if smooth_w is not None else None
    sd = to_device(s.detach(), dev, torch.float32)
    _lib.call("llmc_scale_apply", C.c_void_p(ctx(dev)), _lib.ptr(sd), _lib.ptr(sw),
              _lib.dtype_code(sw.dtype) if sw is not None else 0, _lib.ptr(bw), _lib.dtype_code(bw.dtype),
              C.c_int64(bw.shape[0]), C.c_int64(bw.shape[1]))
    return sw, bw


class AWQModifier(ModifierBase):
    """Collects activation absmax per mapping (like SmoothQuant), then at OnEnd searches
    and applies the per-channel scale of every mapping."""

    def __init__(self, config: AWQConfig):
        if config is None:
            raise ArgumentError("config must not be null")
        super().__init__("AWQ", config.targets, config.ignore)
        self.config = config
        self._running: dict[str, torch.Tensor] = {}
        self.chosen: dict[str, int] = {}

    def on_initialize(self, state):
        self._running.clear()

    def on_batch_core(self, state):
        if state.layer_activations is None:
            return
        for mp in self.config.mappings:
            x = state.layer_activations.get(mp.activation_key)
            if x is not None:
                self._running[mp.activation_key] = act_absmax(x, self._running.get(mp.activation_key))

    def on_end_core(self, state):
        for mp in self.config.mappings:
            mp: SmoothQuantMapping
            if mp.activation_key not in self._running:
                x = state.layer_activations.get(mp.activation_key) if state.layer_activations else None
                if x is None:
                    raise InvalidOperationError(f"AWQ: no activation collected for '{mp.activation_key}'.")
                self._running[mp.activation_key] = act_absmax(x)
            bw = state.named_weights[mp.balance_weight]
            s, k, _ = awq_search(bw, self._running[mp.activation_key], self.config.n_grid, self.config.quant())
            self.chosen[mp.balance_weight] = k
            sw = state.named_weights.get(mp.smooth_weight) if mp.smooth_weight else None
            new_s, new_b = scale_apply(sw, bw, s)
            state.named_weights[mp.balance_weight] = new_b if bw.is_cuda else new_b.cpu()
            if sw is not None:
                state.named_weights[mp.smooth_weight] = new_s if sw.is_cuda else new_s.cpu()
