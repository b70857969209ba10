"""Hessian accumulation and damped Cholesky inverse on the B200.

Mirrors ``HessianAccumulator`` (src/LLMCompressorSharp.TorchExtensions/Hessian/
HessianAccumulator.cs:16-99), ``HessianInverseSolver`` (HessianInverseSolver.cs:25-108)
and ``ActivationHookManager`` (ActivationHookManager.cs:18-85).
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._device import DeviceView, ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, ArgumentOutOfRangeError, ShapeError


class HessianAccumulator:
    """H = sum X^T X (fp32, device-resident) over every Update call."""

    def __init__(self, in_features: int, device: torch.device | str | None = None):
        if in_features <= 0:
            raise ArgumentOutOfRangeError(f"inFeatures must be positive (got {in_features}).")
        self.in_features = int(in_features)
        self.device = torch.device(device) if device is not None else target_device()
        self._ctx = ctx(self.device)
        h = C.c_void_p()
        _lib.call("llmc_hessian_create", C.c_void_p(self._ctx), C.c_int64(in_features), C.byref(h))
        self._h = h.value

    # HessianAccumulator.cs:38
    @property
    def sample_count(self) -> int:
        v = C.c_int64()
        _lib.call("llmc_hessian_sample_count", C.c_void_p(self._require()), C.byref(v))
        return int(v.value)

    def _require(self) -> int:
        if self._h is None:
            raise ArgumentError("HessianAccumulator has been disposed")
        return self._h

    def update(self, x: torch.Tensor) -> None:
        """HessianAccumulator.Update (:47-67): flattens leading dims and adds X^T X."""
        if x is None:
            raise ArgumentError("x must not be null")
        h = self._require()
        if x.dim() == 0 or x.shape[-1] != self.in_features:
            last = x.shape[-1] if x.dim() else None
            raise ShapeError(f"Input last dim ({last}) must equal inFeatures ({self.in_features}).")
        xd = to_device(supported_dtype(x.detach()), self.device).reshape(-1, self.in_features)
        _lib.ctx_for(self.device.index)
        _lib.call("llmc_hessian_update", C.c_void_p(h), _lib.ptr(xd), _lib.dtype_code(xd.dtype),
                  C.c_int64(xd.shape[0]), C.c_int64(self.in_features))

    def get_hessian(self) -> torch.Tensor:
        """GetHessian (:71-75): full symmetric fp32 copy on the device."""
        out = torch.empty(self.in_features, self.in_features, dtype=torch.float32, device=self.device)
        _lib.ctx_for(self.device.index)
        _lib.call("llmc_hessian_get", C.c_void_p(self._require()), _lib.ptr(out))
        return out

    def raw(self) -> torch.Tensor:
        """Zero-copy view of the accumulator (upper triangle authoritative)."""
        p = C.c_void_p()
        _lib.call("llmc_hessian_data", C.c_void_p(self._require()), C.byref(p))
        return torch.as_tensor(DeviceView(p.value, (self.in_features, self.in_features)), device=self.device)

    def add_samples(self, rows: int) -> None:
        _lib.call("llmc_hessian_add_samples", C.c_void_p(self._require()), C.c_int64(rows))

    def reset(self) -> None:
        """Reset (:78-83)."""
        _lib.ctx_for(self.device.index)
        _lib.call("llmc_hessian_reset", C.c_void_p(self._require()))

    def dispose(self) -> None:
        if getattr(self, "_h", None) is not None:
            _lib.call("llmc_hessian_destroy", C.c_void_p(self._h))
            self._h = None

    close = dispose

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


class HessianInverseSolver:
    """HessianInverseSolver.Compute (:44-108) on the device."""

    @staticmethod
    def compute(hessian: torch.Tensor, damping_frac: float) -> torch.Tensor:
        """(H + damp*mean(diag H)*I)^-1; pinv of that matrix when it has no Cholesky factor (:85-91)."""
        return _chol(hessian, damping_frac, want_upper=False)

    @staticmethod
    def upper(hessian: torch.Tensor, damping_frac: float, upper_only: bool = False) -> torch.Tensor:
        """U with U^T U = (H + damp*mean(diag H)*I)^-1 in one factorisation (the factor GPTQ needs).
        Without a Cholesky factor: GPTQ's factor of the pinv fallback, chol(Hinv)^T or Hinv itself
        (GptqBlockQuantizer.cs:105-118)."""
        return _chol(hessian, damping_frac, want_upper=True, upper_only=upper_only)


def _chol(hessian, damping_frac, want_upper, upper_only=False):
    if hessian is None:
        raise ArgumentError("hessian must not be null")
    if hessian.dim() != 2 or hessian.shape[0] != hessian.shape[1]:
        raise ShapeError(f"Hessian must be a square 2-D tensor; got shape {list(hessian.shape)}.")
    dev = target_device(hessian)
    h = to_device(hessian.detach(), dev, torch.float32)
    d = h.shape[0]
    out = torch.empty(d, d, dtype=torch.float32, device=dev)
    _lib.call("llmc_chol_inverse", C.c_void_p(ctx(dev)), _lib.ptr(h), C.c_int64(d), C.c_int64(d),
              C.c_float(damping_frac), int(upper_only), _lib.ptr(out), C.c_int64(d), int(want_upper))
    return out if hessian.is_cuda else out.cpu()


def upper_factor(hinv: torch.Tensor) -> torch.Tensor:
    """U = chol(Hinv)^T with the Hinv fallback (GptqBlockQuantizer.cs:105-118)."""
    dev = target_device(hinv)
    h = to_device(hinv.detach(), dev, torch.float32)
    d = h.shape[0]
    out = torch.empty(d, d, dtype=torch.float32, device=dev)
    _lib.call("llmc_upper_factor", C.c_void_p(ctx(dev)), _lib.ptr(h), C.c_int64(d), C.c_int64(d), _lib.ptr(out),
              C.c_int64(d))
    return out


class ForwardHookHandle:
    """ForwardHookHandle.cs:14-33 — disposing removes the hook (idempotent).  ``remover`` is the
    removal action: a callable, or torch's hook handle (its ``remove``)."""

    def __init__(self, remover):
        if remover is None:
            raise ArgumentError("remove action must not be null")
        self._remover = remover

    def dispose(self):
        if self._remover is not None:
            r, self._remover = self._remover, None
            if callable(r):
                r()
            else:
                r.remove()


class ActivationHookManager:
    """ActivationHookManager.cs:18-85: forward hooks that feed each module's input to its
    accumulator.  (torch fires forward hooks on every module call, including the
    sub-module calls inside a full model's forward.)"""

    def __init__(self):
        self._handles: list[ForwardHookHandle] = []
        self._disposed = False

    def register_for(self, layer: torch.nn.Module, accumulator: HessianAccumulator) -> ForwardHookHandle:
        if layer is None or accumulator is None:
            raise ArgumentError("layer and accumulator must not be null")
        if self._disposed:
            raise ArgumentError("ActivationHookManager has been disposed")

        def hook(mod, inputs, output):
            accumulator.update(inputs[0])
            return output

        h = ForwardHookHandle(layer.register_forward_hook(hook))
        self._handles.append(h)
        return h

    def clear(self):
        for h in self._handles:
            h.dispose()
        self._handles.clear()

    def dispose(self):
        if not self._disposed:
            self.clear()
            self._disposed = True
