"""SparseGPT on the B200 (the reference plans it in
docs/superpowers/plans/2026-05-18-phase-4c-sparsegpt.md; this follows that plan's mask rules
in the U-factor column loop that GptqBlockQuantizer.cs:124-181 uses for GPTQ)."""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._device import ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, InvalidOperationError
from .hessian import ActivationHookManager, HessianAccumulator, HessianInverseSolver
from .session import ModifierBase


@dataclass
class SparseGPTConfig:
    sparsity: float = 0.5
    mask_structure: str = "unstructured"  # "unstructured" or "N:M", e.g. "2:4"
    block_size: int = 128
    dampening_frac: float = 0.01
    targets: list = field(default_factory=list)
    ignore: list = field(default_factory=list)
    type: str = "SparseGPT"

    def nm(self):
        if self.mask_structure in ("", "unstructured", "0:0"):
            return 0, 0
        n, m = self.mask_structure.split(":")
        return int(n), int(m)

    def to_c(self) -> _lib.QConfig:
        n, m = self.nm()
        return _lib.QConfig(num_bits=8, symmetric=1, strategy=0, block_size=self.block_size,
                            damp=self.dampening_frac, sparsity=self.sparsity, mask_n=n, mask_m=m)


def sparsegpt_prune_u(weight: torch.Tensor, upper: torch.Tensor, config: SparseGPTConfig):
    """Returns (pruned fp32 weight, keep mask uint8) on the device."""
    dev = target_device(weight, upper)
    w = to_device(supported_dtype(weight.detach()), dev)
    u = to_device(upper.detach(), dev, torch.float32)
    m, n = w.shape
    out = torch.empty(m, n, dtype=torch.float32, device=dev)
    mask = torch.empty(m, n, dtype=torch.uint8, device=dev)
    cfg = config.to_c()
    _lib.call("llmc_sparsegpt_prune", C.c_void_p(ctx(dev)), _lib.ptr(w), _lib.dtype_code(w.dtype), C.c_int64(m),
              C.c_int64(n), C.c_int64(n), _lib.ptr(u), C.c_int64(n), C.byref(cfg), _lib.ptr(out), C.c_int64(n),
              _lib.ptr(mask))
    return out, mask


class SparseGPTModifier(ModifierBase):
    """Calibration hooks as GPTQModifier; OnEnd prunes each targeted weight and writes it
    back in its original dtype (plan :1652-1655)."""

    def __init__(self, config: SparseGPTConfig):
        if config is None:
            raise ArgumentError("config must not be null")
        super().__init__("SparseGPT", config.targets, config.ignore)
        self.config = config
        self._hooks = None
        self._acc = None

    def on_initialize(self, state):
        pass

    def on_start_core(self, state):
        if state.named_modules is None:
            raise InvalidOperationError("SparseGPTModifier requires CompressionState.NamedModules to be populated.")
        self._hooks = ActivationHookManager()
        self._acc = {}
        for wname in self.targeted_names(state):
            lname = wname[: -len(".weight")] if wname.endswith(".weight") else wname
            module = state.named_modules.get(lname)
            if module is None:
                continue
            acc = HessianAccumulator(state.named_weights[wname].shape[-1], target_device(state.named_weights[wname]))
            self._acc[wname] = acc
            self._hooks.register_for(module, acc)

    def on_end_core(self, state):
        if self._hooks is not None:
            self._hooks.dispose()
            self._hooks = None
        for wname, acc in (self._acc or {}).items():
            if acc.sample_count == 0:  # plan :1559-1567: no calibration data -> weight unchanged
                continue
            u = HessianInverseSolver.upper(acc.raw(), self.config.dampening_frac, upper_only=True)
            w = state.named_weights[wname]
            out, mask = sparsegpt_prune_u(w, u, self.config)
            res = out.to(w.dtype)
            state.named_weights[wname] = res if w.is_cuda else res.cpu()
            state.compressed[wname] = {"mask": mask}

    def on_finalize_core(self, state):
        if self._hooks is not None:
            self._hooks.dispose()
        for a in (self._acc or {}).values():
            a.dispose()
        self._acc = None
