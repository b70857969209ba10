"""Fake quantisation, observers and int4 packing on the B200.

Mirrors ``FakeQuantize`` (src/LLMCompressorSharp.TorchExtensions/Quantization/FakeQuantize.cs:22-38,
FakeQuantizeFunction.cs:30-68), ``Int4PackedTensor`` (Int4PackedTensor.cs:17-162) and the
observer family (Observers/Observer.cs:17-75, MinMaxObserver.cs:14-71,
PerChannelMinMaxObserver.cs:15-112, MovingAverageMinMaxObserver.cs:16-88) plus a
group observer (one min/max per (row, group) of a 2-D weight).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._device import ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, ArgumentOutOfRangeError, InvalidOperationError

f32 = np.float32


def _check_bits(num_bits: int):
    if num_bits < 2 or num_bits > 16:
        raise ArgumentOutOfRangeError(f"numBits must be between 2 and 16 inclusive (got {num_bits}).")


class _FakeQuantizeFn(torch.autograd.Function):
    """Forward on the device; backward is the straight-through estimator
    (FakeQuantizeFunction.cs:56-68)."""

    @staticmethod
    def forward(ctx_, x, scale, zp, num_bits, symmetric):
        dev = target_device(x)
        xd = to_device(supported_dtype(x.detach()), dev)
        out = torch.empty_like(xd)
        _lib.call("llmc_fake_quantize", C.c_void_p(ctx(dev)), _lib.ptr(xd), _lib.dtype_code(xd.dtype),
                  C.c_int64(xd.numel()), C.c_float(scale), C.c_int32(int(zp)), C.c_int32(num_bits),
                  C.c_int32(int(symmetric)), _lib.ptr(out), C.c_void_p(0))
        out = out.reshape(x.shape)
        return out if x.is_cuda else out.cpu()

    @staticmethod
    def backward(ctx_, grad):
        return grad, None, None, None, None


class FakeQuantize:
    @staticmethod
    def apply(x: torch.Tensor, scale: float, zero_point: int, num_bits: int, symmetric: bool) -> torch.Tensor:
        if x is None:
            raise ArgumentError("x must not be null")
        _check_bits(num_bits)
        return _FakeQuantizeFn.apply(x, float(scale), int(zero_point), int(num_bits), bool(symmetric))


def affine_params(mins: torch.Tensor, maxs: torch.Tensor, num_bits: int, symmetric: bool):
    """Observer.ComputeAffineParams (Observer.cs:47-75) element-wise on the device."""
    _check_bits(num_bits)
    dev = target_device(mins, maxs)
    mn = to_device(mins.detach().reshape(-1), dev, torch.float32)
    mx = to_device(maxs.detach().reshape(-1), dev, torch.float32)
    s = torch.empty_like(mn)
    z = torch.empty(mn.shape, dtype=torch.int32, device=dev)
    _lib.call("llmc_affine_params", C.c_void_p(ctx(dev)), _lib.ptr(mn), _lib.ptr(mx), C.c_int64(mn.numel()),
              C.c_int32(num_bits), C.c_int32(int(symmetric)), _lib.ptr(s), _lib.ptr(z))
    return s.reshape(mins.shape), z.reshape(mins.shape)


def _minmax(x: torch.Tensor, strategy: int, group_size: int, mins, maxs, accumulate: bool):
    dev = mins.device
    xd = to_device(supported_dtype(x.detach()), dev)
    x2 = xd.reshape(xd.shape[0], -1) if xd.dim() >= 2 else xd.reshape(1, -1)
    _lib.call("llmc_observer_minmax", C.c_void_p(ctx(dev)), _lib.ptr(x2), _lib.dtype_code(x2.dtype),
              C.c_int64(x2.shape[0]), C.c_int64(x2.shape[1]), C.c_int64(x2.shape[1]), C.c_int32(strategy),
              C.c_int64(group_size), _lib.ptr(mins), _lib.ptr(maxs), C.c_int32(int(accumulate)))


class Observer:
    """Observer.cs:17-75."""

    strategy = "tensor"

    def update(self, x: torch.Tensor) -> None:
        raise NotImplementedError

    def get_quant_params(self, num_bits: int, symmetric: bool):
        raise NotImplementedError

    def reset(self) -> None:
        raise NotImplementedError


class MinMaxObserver(Observer):
    """MinMaxObserver.cs:14-71; the running min/max stays on the device."""

    strategy = "tensor"

    def __init__(self, device=None):
        self.device = torch.device(device) if device is not None else None
        self.reset()

    def update(self, x: torch.Tensor) -> None:
        if x is None:
            raise ArgumentError("x must not be null")
        if self.device is None:
            self.device = target_device(x)
        if self._mm is None:
            # MinMaxObserver.cs:16-17: the running values start at +inf / -inf, and every batch
            # is folded in by the observer's strict-less rule (a batch holding a NaN changes
            # nothing, MinMaxObserver.cs:34-42).
            self._mm = torch.tensor([float("inf"), float("-inf")], dtype=torch.float32, device=self.device)
        _minmax(x, 0, 0, self._mm[0:1], self._mm[1:2], True)
        self._has = True

    def get_quant_params(self, num_bits: int, symmetric: bool):
        if not self._has:
            raise InvalidOperationError("MinMaxObserver has no calibration samples. Call Update before GetQuantParams.")
        s, z = affine_params(self._mm[0:1], self._mm[1:2], num_bits, symmetric)
        return float(s.item()), int(z.item())

    def min_max(self):
        return float(self._mm[0].item()), float(self._mm[1].item())

    def reset(self) -> None:
        self._mm = None
        self._has = False


class PerChannelMinMaxObserver(Observer):
    """PerChannelMinMaxObserver.cs:15-112 (any rank; statistics per index along the axis)."""

    strategy = "channel"

    def __init__(self, channel_axis: int = 0, device=None):
        self.channel_axis = channel_axis
        self.device = torch.device(device) if device is not None else None
        self.reset()

    def update(self, x: torch.Tensor) -> None:
        if x is None:
            raise ArgumentError("x must not be null")
        if self.channel_axis < 0 or self.channel_axis >= x.dim():
            raise ArgumentOutOfRangeError(
                f"channelAxis {self.channel_axis} is out of range for tensor of rank {x.dim()}.")
        if self.device is None:
            self.device = target_device(x)
        xt = x.movedim(self.channel_axis, 0) if self.channel_axis else x
        c = xt.shape[0]
        if self._min is None:
            self._min = torch.empty(c, dtype=torch.float32, device=self.device)
            self._max = torch.empty(c, dtype=torch.float32, device=self.device)
            acc = False
        else:
            acc = True
        _minmax(xt.reshape(c, -1), 1, 0, self._min, self._max, acc)

    def get_quant_params(self, num_bits: int, symmetric: bool):
        if self._min is None:
            raise InvalidOperationError(
                "PerChannelMinMaxObserver has no calibration samples. Call Update before GetQuantParams.")
        return affine_params(self._min, self._max, num_bits, symmetric)

    def reset(self) -> None:
        self._min = None
        self._max = None


class GroupMinMaxObserver(Observer):
    """One min/max per (row, group of ``group_size`` columns) of a 2-D weight (extension;
    the reference has no group strategy)."""

    strategy = "group"

    def __init__(self, group_size: int = 128, device=None):
        self.group_size = group_size
        self.device = torch.device(device) if device is not None else None
        self.reset()

    def update(self, x: torch.Tensor) -> None:
        if self.device is None:
            self.device = target_device(x)
        m, n = x.shape
        g = (n + self.group_size - 1) // self.group_size
        if self._min is None:
            self._min = torch.empty(m, g, dtype=torch.float32, device=self.device)
            self._max = torch.empty(m, g, dtype=torch.float32, device=self.device)
            acc = False
        else:
            acc = True
        _minmax(x, 3, self.group_size, self._min, self._max, acc)

    def get_quant_params(self, num_bits: int, symmetric: bool):
        if self._min is None:
            raise InvalidOperationError("GroupMinMaxObserver has no calibration samples.")
        return affine_params(self._min, self._max, num_bits, symmetric)

    def reset(self) -> None:
        self._min = None
        self._max = None


class MovingAverageMinMaxObserver(Observer):
    """MovingAverageMinMaxObserver.cs:16-88: device min/max per batch, EMA of the two
    scalars in C# float arithmetic."""

    strategy = "tensor"

    def __init__(self, averaging_constant: float = 0.01, device=None):
        if not (0.0 < averaging_constant <= 1.0):
            raise ArgumentOutOfRangeError("averagingConstant must be in (0, 1].")
        self._alpha = f32(averaging_constant)
        self.device = torch.device(device) if device is not None else None
        self._mm = None
        self.reset()

    def update(self, x: torch.Tensor) -> None:
        if x is None:
            raise ArgumentError("x must not be null")
        if self.device is None:
            self.device = target_device(x)
        if self._mm is None:
            self._mm = torch.empty(2, dtype=torch.float32, device=self.device)
        # The batch's own x.min() / x.max() (MovingAverageMinMaxObserver.cs:44-47), NaN included.
        _minmax(x, 0, 0, self._mm[0:1], self._mm[1:2], False)
        bmin, bmax = (f32(v) for v in self._mm.tolist())
        if not self._has:
            self._min, self._max, self._has = bmin, bmax, True
        else:
            one_m = f32(f32(1) - self._alpha)
            self._min = f32(f32(one_m * self._min) + f32(self._alpha * bmin))
            self._max = f32(f32(one_m * self._max) + f32(self._alpha * bmax))

    def get_quant_params(self, num_bits: int, symmetric: bool):
        if not self._has:
            raise InvalidOperationError("MovingAverageMinMaxObserver has no calibration samples.")
        dev = self.device
        s, z = affine_params(torch.tensor([self._min], device=dev), torch.tensor([self._max], device=dev), num_bits,
                             symmetric)
        return float(s.item()), int(z.item())

    def reset(self) -> None:
        self._min = f32(0)
        self._max = f32(0)
        self._has = False


class MSEObserver(Observer):
    """MSEObserver.cs:17-124: keeps the calibration samples (device copies) and, in
    get_quant_params, grid-searches the symmetric ranges +-absMax*i/G for the (scale, zero-point)
    with the lowest fake-quantisation MSE (llmc_observer_mse: one device pass adds the squared
    errors of every candidate; the candidates and the choice are the reference's scalar math)."""

    strategy = "tensor"

    def __init__(self, grid_points: int = 100, device=None):
        if grid_points < 2:
            raise ArgumentOutOfRangeError("gridPoints must be >= 2.")
        self.grid_points = grid_points
        self.device = torch.device(device) if device is not None else None
        self._samples: list[torch.Tensor] = []
        self.last_mse = None

    def update(self, x: torch.Tensor) -> None:
        if x is None:
            raise ArgumentError("x must not be null")
        if self.device is None:
            self.device = target_device(x)
        self._samples.append(to_device(supported_dtype(x.detach()), self.device).flatten().clone())

    def get_quant_params(self, num_bits: int, symmetric: bool):
        if not self._samples:
            raise InvalidOperationError("MSEObserver has no calibration samples. Call Update before GetQuantParams.")
        _check_bits(num_bits)
        flat = torch.cat(self._samples) if len(self._samples) > 1 else self._samples[0]
        scale, zp = C.c_float(), C.c_int32()
        mse = np.empty(self.grid_points, dtype=np.float64)
        _lib.call("llmc_observer_mse", C.c_void_p(ctx(self.device)), _lib.ptr(flat), _lib.dtype_code(flat.dtype),
                  C.c_int64(flat.numel()), C.c_int32(self.grid_points), C.c_int32(num_bits), C.c_int32(int(symmetric)),
                  C.byref(scale), C.byref(zp), C.c_void_p(mse.ctypes.data))
        self.last_mse = mse
        return float(scale.value), int(zp.value)

    def reset(self) -> None:
        self._samples.clear()
        self.last_mse = None


class Int4PackedTensor:
    """Int4PackedTensor.cs:17-162: codes q - zp stored two per byte, even index in the high
    nibble.  The bytes live on the device."""

    def __init__(self, packed: torch.Tensor, count: int, scale: float, zero_point: int, symmetric: bool):
        self.packed = packed
        self.element_count = count
        self.scale = float(f32(scale))
        self.zero_point = int(zero_point)
        self.symmetric = symmetric

    @staticmethod
    def from_float(x: torch.Tensor, scale: float, zero_point: int, symmetric: bool) -> "Int4PackedTensor":
        """FromFloat (:79-100): integer codes of the 4-bit fake-quant chain, then packed."""
        dev = target_device(x)
        xd = to_device(supported_dtype(x.detach()), dev).reshape(-1)
        n = xd.numel()
        q = torch.empty(n, dtype=torch.int32, device=dev)
        c = C.c_void_p(ctx(dev))
        _lib.call("llmc_fake_quantize", c, _lib.ptr(xd), _lib.dtype_code(xd.dtype), C.c_int64(n),
                  C.c_float(scale), C.c_int32(int(zero_point)), C.c_int32(4), C.c_int32(int(symmetric)),
                  C.c_void_p(0), _lib.ptr(q))
        codes = torch.empty((n + 1) // 2, dtype=torch.uint8, device=dev)
        _lib.call("llmc_int4_pack", c, _lib.ptr(q), C.c_int64(n), C.c_int32(int(zero_point)), _lib.ptr(codes))
        return Int4PackedTensor(codes, n, scale, zero_point, symmetric)

    @property
    def packed_bytes(self) -> bytes:
        return bytes(self.packed.cpu().numpy().tobytes())

    @staticmethod
    def from_packed_bytes(packed, element_count: int, scale: float, zero_point: int, symmetric: bool):
        b = packed if isinstance(packed, torch.Tensor) else torch.frombuffer(bytearray(packed), dtype=torch.uint8)
        if b.numel() != (element_count + 1) // 2:
            raise ArgumentError(
                f"Expected {(element_count + 1) // 2} bytes for {element_count} int4 elements; got {b.numel()}.")
        dev = target_device(b)
        return Int4PackedTensor(to_device(b, dev), element_count, scale, zero_point, symmetric)

    def dequantize(self) -> torch.Tensor:
        """Dequantize (:152-161): stored value * scale (fp32)."""
        dev = self.packed.device
        out = torch.empty(self.element_count, dtype=torch.float32, device=dev)
        _lib.call("llmc_int4_unpack_dequant", C.c_void_p(ctx(dev)), _lib.ptr(self.packed),
                  C.c_int64(self.element_count), C.c_float(self.scale), C.c_int32(self.zero_point),
                  C.c_int32(int(self.symmetric)), _lib.ptr(out))
        return out


def quantize_per_token(x: torch.Tensor, num_bits: int = 8, symmetric: bool = True, want_values: bool = False):
    """Dynamic per-token quantisation of activations x [tokens, hidden] (extension; the reference
    rejects PerToken for weights, RtnModifier.cs:69-70): one min-max observer per token row,
    ComputeAffineParams and the FakeQuantize op chain in x's dtype, on the device
    (llmc_act_quant_per_token).  Returns (codes, scales [tokens] fp32, zero-points [tokens] int32,
    fake-quantised x or None); codes are int8 for a symmetric grid and uint8 otherwise."""
    _check_bits(num_bits)
    if num_bits > 8:
        raise ArgumentOutOfRangeError("per-token codes are bytes: num_bits must be <= 8")
    dev = target_device(x)
    xd = to_device(supported_dtype(x.detach()), dev)
    x2 = xd.reshape(-1, xd.shape[-1]) if xd.dim() != 2 else xd
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows, cols = x2.shape
    codes = torch.empty(rows, cols, dtype=torch.int8 if symmetric else torch.uint8, device=dev)
    scales = torch.empty(rows, dtype=torch.float32, device=dev)
    zps = torch.empty(rows, dtype=torch.int32, device=dev)
    deq = torch.empty(rows, cols, dtype=x2.dtype, device=dev) if want_values else None
    _lib.call("llmc_act_quant_per_token", C.c_void_p(ctx(dev)), _lib.ptr(x2), _lib.dtype_code(x2.dtype),
              C.c_int64(rows), C.c_int64(cols), C.c_int64(x2.stride(0)), C.c_int32(num_bits), C.c_int32(int(symmetric)),
              _lib.ptr(codes), C.c_int64(cols), _lib.ptr(scales), _lib.ptr(zps), _lib.ptr(deq), C.c_int64(cols))
    return codes, scales, zps, deq
