"""SmoothQuant activation statistics and smoothing (oracle; test infrastructure only).

Restates ``SmoothQuantModifier.UpdateActivationMax`` (src/LLMCompressorSharp.Core/
Algorithms/SmoothQuant/SmoothQuantModifier.cs:71-115) and ``ApplyMapping`` (:117-182).
The per-channel smoothing scale is C# float math with ``MathF.Pow``; it is restated
with numpy float32 ``power`` (correctly rounded in practice; see the tolerance notes
in the tests).
"""

from __future__ import annotations

import numpy as np
import torch

f32 = np.float32


def act_absmax(x: torch.Tensor) -> np.ndarray:
    """|x|.amax over all dims but the last, as fp32 (:73-93)."""
    a = x.detach().abs().to(torch.float32)
    if a.dim() == 1:
        return a.numpy().copy()
    return a.reshape(-1, a.shape[-1]).amax(dim=0).numpy()


def update_running_max(running: np.ndarray | None, x: torch.Tensor) -> np.ndarray:
    """Running element-wise max of batch absmax (:94-114)."""
    b = act_absmax(x)
    if running is None:
        return b
    if running.shape != b.shape:
        raise RuntimeError(f"SmoothQuant: activation feature dim changed: expected {running.shape[0]}, got {b.shape[0]}.")
    return np.maximum(running, b)


def smoothing_scales(act_max: np.ndarray, weight_max: np.ndarray, alpha: float) -> np.ndarray:
    """s_i = max(max(a_i,1e-5)^alpha / max(w_i,1e-5)^(1-alpha), 1e-5) (:165-172)."""
    a = np.maximum(act_max.astype(np.float32), f32(1e-5))
    w = np.maximum(weight_max.astype(np.float32), f32(1e-5))
    al = f32(alpha)
    num = np.power(a, al, dtype=np.float32)
    den = np.power(w, f32(f32(1) - al), dtype=np.float32)
    return np.maximum((num / den).astype(np.float32), f32(1e-5)).astype(np.float32)


def apply_mapping(smooth_w: torch.Tensor, balance_w: torch.Tensor, act_max: np.ndarray, alpha: float):
    """ApplyMapping (:117-182).  Returns (new_smooth, new_balance) in the input dtypes."""
    if smooth_w.dim() != 1:
        raise RuntimeError(f"SmoothQuant: smooth weight must be 1-D (got rank {smooth_w.dim()}).")
    if balance_w.dim() != 2:
        raise RuntimeError(f"SmoothQuant: balance weight must be 2-D (got rank {balance_w.dim()}).")
    hidden = smooth_w.shape[0]
    if act_max.shape[0] != hidden:
        raise RuntimeError(f"SmoothQuant: activation hidden dim {act_max.shape[0]} does not match smooth weight {hidden}.")
    if balance_w.shape[1] != hidden:
        raise RuntimeError(f"SmoothQuant: balance weight last dim {balance_w.shape[1]} does not match hidden {hidden}.")
    wmax = balance_w.abs().amax(dim=0).to(torch.float32).numpy()  # :160-162
    s = smoothing_scales(act_max, wmax, alpha)
    scale = torch.from_numpy(s).to(smooth_w.dtype)  # tensor(s).to(smoothW.dtype), :174
    new_smooth = smooth_w.div(scale)  # :175
    new_balance = balance_w.mul(scale)  # :178
    return new_smooth, new_balance, s
