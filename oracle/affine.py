"""Observers and affine-parameter math (oracle; test infrastructure only).

Restates:
  * ``Observer.ComputeAffineParams``  src/LLMCompressorSharp.TorchExtensions/Observers/Observer.cs:47-75
  * ``MinMaxObserver``                src/LLMCompressorSharp.TorchExtensions/Observers/MinMaxObserver.cs:14-71
  * ``PerChannelMinMaxObserver``      src/LLMCompressorSharp.TorchExtensions/Observers/PerChannelMinMaxObserver.cs:15-112
  * ``MovingAverageMinMaxObserver``   src/LLMCompressorSharp.TorchExtensions/Observers/MovingAverageMinMaxObserver.cs:16-88
  * ``MSEObserver``                   src/LLMCompressorSharp.TorchExtensions/Observers/MSEObserver.cs:17-124

C# ``float`` scalar arithmetic is restated with ``numpy.float32`` (IEEE single, one
rounding per operation, as RyuJIT's SSE code does) and ``MathF.Round`` with
``numpy.rint`` (round half to even).
"""

from __future__ import annotations

import numpy as np
import torch

f32 = np.float32


def compute_affine_params(mn: float, mx: float, num_bits: int, symmetric: bool) -> tuple[float, int]:
    """Observer.ComputeAffineParams, Observer.cs:47-75.

    Symmetric: scale = absMax / (2^(b-1)-1) (1 when absMax == 0), zp = 0.
    Asymmetric: scale = (max-min) / (2^b - 1) (1 when the range is 0),
    zp = clamp((long)MathF.Round(0 - min/scale), 0, 2^b - 1).  The range does not
    include zero (unlike upstream llm-compressor).
    """
    if num_bits < 2 or num_bits > 16:
        raise ValueError("numBits must be between 2 and 16 inclusive.")  # Observer.cs:53-56
    mn = f32(mn)
    mx = f32(mx)
    if symmetric:
        # MathF.Max(MathF.Abs(min), MathF.Abs(max)), :60; MathF.Max returns NaN when either
        # operand is NaN (Python's max would depend on the argument order).
        abs_max = f32(np.nan) if (np.isnan(mn) or np.isnan(mx)) else max(abs(mn), abs(mx))
        q_max = (1 << (num_bits - 1)) - 1
        scale = f32(1.0) if abs_max == f32(0) else f32(abs_max / f32(q_max))
        return float(scale), 0
    q_min = 0
    q_max = (1 << num_bits) - 1
    rng = f32(mx - mn)  # :69
    scale = f32(1.0) if rng == f32(0) else f32(rng / f32(q_max - q_min))  # :70
    with np.errstate(invalid="ignore", divide="ignore"):
        zf = np.rint(f32(f32(q_min) - f32(mn / scale)))  # :71, MathF.Round = half-even
    # (long) of a float saturates in .NET 10 (the reference's target): NaN -> 0, +-inf -> the
    # long range; Math.Clamp then bounds it (:72).
    zp = 0 if np.isnan(zf) else int(min(max(zf, q_min), q_max))
    return float(scale), zp


def affine_params_array(mins, maxs, num_bits: int, symmetric: bool):
    """Vectorised ComputeAffineParams over arrays of (min, max); element-wise identical
    to the scalar loop in PerChannelMinMaxObserver.GetQuantParams (:93-96)."""
    mins = np.asarray(mins, dtype=np.float32)
    maxs = np.asarray(maxs, dtype=np.float32)
    if num_bits < 2 or num_bits > 16:
        raise ValueError("numBits must be between 2 and 16 inclusive.")
    with np.errstate(divide="ignore", invalid="ignore"):
        if symmetric:
            q_max = f32((1 << (num_bits - 1)) - 1)
            abs_max = np.maximum(np.abs(mins), np.abs(maxs))
            scale = np.where(abs_max == 0, f32(1), (abs_max / q_max).astype(np.float32)).astype(np.float32)
            zp = np.zeros(scale.shape, dtype=np.int64)
            return scale, zp
        q_max = (1 << num_bits) - 1
        rng = (maxs - mins).astype(np.float32)
        scale = np.where(rng == 0, f32(1), (rng / f32(q_max)).astype(np.float32)).astype(np.float32)
        zf = np.rint((f32(0) - (mins / scale).astype(np.float32)).astype(np.float32))
        zp = np.where(np.isnan(zf), 0, np.clip(zf, 0, q_max)).astype(np.int64)  # saturating, NaN -> 0
        return scale, zp


def observer_fold(b_min, b_max):
    """MinMaxObserver.Update on a new observer (MinMaxObserver.cs:16-17,34-42): the running
    values start at +inf / -inf and take the batch value only when it is strictly beyond them,
    so a NaN batch minimum (torch's x.min() of a tensor holding a NaN) leaves +inf.  Works on
    scalars and, element-wise, on arrays (one observer per element, as ComputeScaleZeroPoint
    creates one per row, GptqBlockQuantizer.cs:212-230)."""
    b_min = np.asarray(b_min, dtype=np.float32)
    b_max = np.asarray(b_max, dtype=np.float32)
    with np.errstate(invalid="ignore"):
        mn = np.where(b_min < np.float32(np.inf), b_min, np.float32(np.inf)).astype(np.float32)
        mx = np.where(b_max > np.float32(-np.inf), b_max, np.float32(-np.inf)).astype(np.float32)
    return mn, mx


def _as_f32(x: torch.Tensor) -> torch.Tensor:
    # The reference reads statistics back with item<float>()/data<float>().  Upcasting a
    # bf16/fp16 min or max to fp32 is exact, so doing it before the reduction is lossless.
    return x.detach().to(torch.float32)


class MinMaxObserver:
    """MinMaxObserver.cs:14-71 — running global min/max, per-tensor params."""

    strategy = "tensor"

    def __init__(self):
        self.reset()

    def update(self, x: torch.Tensor) -> None:  # :24-45
        xf = _as_f32(x)
        b_min = f32(xf.min().item())
        b_max = f32(xf.max().item())
        if b_min < self._min:
            self._min = b_min
        if b_max > self._max:
            self._max = b_max
        self._has = True

    def get_quant_params(self, num_bits: int, symmetric: bool):  # :48-62
        if not self._has:
            raise RuntimeError("MinMaxObserver has no calibration samples. Call Update before GetQuantParams.")
        return compute_affine_params(self._min, self._max, num_bits, symmetric)

    def reset(self) -> None:  # :65-70
        self._min = f32(np.inf)
        self._max = f32(-np.inf)
        self._has = False


class PerChannelMinMaxObserver:
    """PerChannelMinMaxObserver.cs:15-112 — running per-channel min/max along one axis."""

    strategy = "channel"

    def __init__(self, channel_axis: int = 0):
        self.channel_axis = channel_axis
        self._min = None
        self._max = None

    def update(self, x: torch.Tensor) -> None:  # :38-76
        if self.channel_axis < 0 or self.channel_axis >= x.dim():
            raise IndexError(f"channelAxis {self.channel_axis} is out of range for tensor of rank {x.dim()}.")
        xf = _as_f32(x)
        dims = [i for i in range(x.dim()) if i != self.channel_axis]
        b_min = xf.amin(dim=dims) if dims else xf.clone()
        b_max = xf.amax(dim=dims) if dims else xf.clone()
        if self._min is None:
            self._min, self._max = b_min.clone(), b_max.clone()
        else:
            self._min = torch.minimum(self._min, b_min)
            self._max = torch.maximum(self._max, b_max)

    def get_quant_params(self, num_bits: int, symmetric: bool):  # :79-102
        if self._min is None:
            raise RuntimeError("PerChannelMinMaxObserver has no calibration samples. Call Update before GetQuantParams.")
        return affine_params_array(self._min.numpy(), self._max.numpy(), num_bits, symmetric)

    def reset(self) -> None:
        self._min = None
        self._max = None


class MovingAverageMinMaxObserver:
    """MovingAverageMinMaxObserver.cs:16-88 — EMA of per-batch min/max."""

    strategy = "tensor"

    def __init__(self, averaging_constant: float = 0.01):
        if not (0.0 < averaging_constant <= 1.0):
            raise ValueError("averagingConstant must be in (0, 1].")
        self._alpha = f32(averaging_constant)
        self.reset()

    def update(self, x: torch.Tensor) -> None:  # :42-62
        xf = _as_f32(x)
        b_min = f32(xf.min().item())
        b_max = f32(xf.max().item())
        if not self._has:
            self._min, self._max, self._has = b_min, b_max, True
        else:
            one_m = f32(f32(1) - self._alpha)
            self._min = f32(f32(one_m * self._min) + f32(self._alpha * b_min))
            self._max = f32(f32(one_m * self._max) + f32(self._alpha * b_max))

    def get_quant_params(self, num_bits: int, symmetric: bool):
        if not self._has:
            raise RuntimeError("MovingAverageMinMaxObserver has no calibration samples.")
        return compute_affine_params(self._min, self._max, num_bits, symmetric)

    def reset(self) -> None:
        self._min = f32(0)
        self._max = f32(0)
        self._has = False


class MSEObserver:
    """MSEObserver.cs:17-124 — grid search over symmetric ranges ±absMax·i/G."""

    strategy = "tensor"

    def __init__(self, grid_points: int = 100):
        if grid_points < 2:
            raise ValueError("gridPoints must be >= 2.")
        self.grid_points = grid_points
        self._samples: list[torch.Tensor] = []

    def update(self, x: torch.Tensor) -> None:
        self._samples.append(x.detach().cpu().clone())

    def get_quant_params(self, num_bits: int, symmetric: bool):  # :50-93
        if not self._samples:
            raise RuntimeError("MSEObserver has no calibration samples.")
        flat = torch.cat([s.flatten() for s in self._samples])
        abs_max = f32(flat.abs().max().item())
        if abs_max == 0:
            return 1.0, 0
        best_scale = f32(abs_max / f32((1 << (num_bits - 1)) - 1))
        best_zp = 0
        best_mse = np.inf
        for i in range(1, self.grid_points + 1):
            frac = f32(f32(i) / f32(self.grid_points))
            cmax = f32(abs_max * frac)
            scale, zp = compute_affine_params(-cmax, cmax, num_bits, symmetric)
            if scale == 0:
                continue
            qmin = -((1 << (num_bits - 1)) - 1) if symmetric else 0
            qmax = (1 << (num_bits - 1)) - 1 if symmetric else (1 << num_bits) - 1
            q = (flat / scale).round_() + zp
            q.clamp_(qmin, qmax)
            fq = (q - zp) * scale
            mse = f32((flat - fq).pow(2).mean().item())
            if mse < best_mse:
                best_mse, best_scale, best_zp = mse, f32(scale), zp
        return float(best_scale), best_zp

    def reset(self) -> None:
        self._samples.clear()


def group_minmax(w: torch.Tensor, group_size: int):
    """Per-(row, column-group) min/max of a 2-D weight.  Extension: the reference has
    no group strategy (QuantizationStrategy.cs:9-19).  It applies the MinMaxObserver
    rule of ComputeScaleZeroPoint (GptqBlockQuantizer.cs:196-234) to every
    (row, group) slice; the last group may be ragged.  Parity unpinned."""
    wf = _as_f32(w)
    m, n = wf.shape
    ng = (n + group_size - 1) // group_size
    mins = torch.empty(m, ng)
    maxs = torch.empty(m, ng)
    for g in range(ng):
        sl = wf[:, g * group_size:min(n, (g + 1) * group_size)]
        mins[:, g] = sl.amin(dim=1)
        maxs[:, g] = sl.amax(dim=1)
    return mins, maxs
