"""Round-to-nearest weight quantisation (oracle; test infrastructure only).

Restates ``RtnModifier.OnEndCore`` / ``ApplyFakeQuant`` / ``ApplyPerChannelFakeQuant``
(src/LLMCompressorSharp.Core/Algorithms/Rtn/RtnModifier.cs:44-122) with the
``RtnConfig`` defaults (Configs/RtnConfig.cs:17-26).  The group strategy is an
extension (no such strategy in QuantizationStrategy.cs:9-19): one MinMax observer per
(row, group) slice.  The fake-quantised output stays in the weight's dtype (:212-213).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .affine import MinMaxObserver, PerChannelMinMaxObserver, affine_params_array, group_minmax
from .fakequant import fake_quantize_codes


@dataclass
class RtnConfig:
    num_bits: int = 8
    symmetric: bool = True
    strategy: str = "tensor"  # 'tensor' | 'channel' | 'group' ('token' raises, :69-70)
    channel_axis: int = 0
    group_size: int = 128


def rtn_params(w: torch.Tensor, cfg: RtnConfig):
    """Observer -> GetQuantParams (:51-54).  Returns (scales, zps) as [m, G] arrays."""
    if cfg.strategy == "tensor":
        obs = MinMaxObserver()
        obs.update(w)
        s, z = obs.get_quant_params(cfg.num_bits, cfg.symmetric)
        rows = w.shape[0] if w.dim() >= 1 else 1
        return np.full((rows, 1), s, np.float32), np.full((rows, 1), z, np.int64)
    if cfg.strategy == "channel":
        obs = PerChannelMinMaxObserver(cfg.channel_axis)
        obs.update(w)
        s, z = obs.get_quant_params(cfg.num_bits, cfg.symmetric)
        return s.reshape(-1, 1), z.reshape(-1, 1)
    if cfg.strategy == "group":
        mins, maxs = group_minmax(w, cfg.group_size)
        return affine_params_array(mins.numpy(), maxs.numpy(), cfg.num_bits, cfg.symmetric)
    if cfg.strategy == "token":
        raise NotImplementedError("PerToken strategy applies to activations, not weights.")
    raise ValueError(f"Unsupported quantization strategy {cfg.strategy}")


def expand_params(scales, zps, n: int, group_size: int):
    """Broadcast [m, G] parameters to [m, n] element parameters."""
    s = torch.from_numpy(np.asarray(scales, np.float32))
    z = torch.from_numpy(np.asarray(zps).astype(np.float32))
    if s.shape[1] == 1:
        return s, z
    col_group = torch.arange(n) // group_size
    return s[:, col_group], z[:, col_group]


def rtn_quantize(w: torch.Tensor, cfg: RtnConfig):
    """Returns (fake-quant in w.dtype, codes int32, scales [m,G], zps [m,G])."""
    if w.dim() == 1:
        # 1-D weights: per-tensor only in practice (RtnModifierTests.cs:22-49).
        out, codes, s, z = rtn_quantize(w.reshape(1, -1), cfg)
        return out.reshape(-1), codes.reshape(-1), s, z
    if cfg.strategy == "channel" and cfg.channel_axis != 0:
        raise NotImplementedError("the 2-D RTN path quantises output channels (axis 0)")
    scales, zps = rtn_params(w, cfg)
    s, z = expand_params(scales, zps, w.shape[1], cfg.group_size)
    out, codes = fake_quantize_codes(w, s, z, cfg.num_bits, cfg.symmetric)
    return out, codes, scales, zps
