"""Dynamic per-token activation quantisation (oracle; test infrastructure only).

Extension, parity unpinned: the reference has QuantizationStrategy.PerToken
(src/LLMCompressorSharp.TorchExtensions/Observers/QuantizationStrategy.cs:9-19) but rejects it
for weights (src/LLMCompressorSharp.Core/Algorithms/Rtn/RtnModifier.cs:69-70) and quantises no
activations.  Restated from the reference's own pieces: one PerChannelMinMaxObserver per token
row (PerChannelMinMaxObserver.cs:38-102 on axis 0 of [tokens, hidden]), ComputeAffineParams
(Observer.cs:47-75) and the FakeQuantizeFunction op chain in x's dtype
(FakeQuantizeFunction.cs:39-44).
"""

from __future__ import annotations

import numpy as np
import torch

from .affine import PerChannelMinMaxObserver
from .fakequant import fake_quantize_codes


def quantize_per_token(x: torch.Tensor, num_bits: int = 8, symmetric: bool = True):
    """x [tokens, hidden] -> (fake-quantised x in x.dtype, codes int32 [tokens, hidden],
    scales fp32 [tokens], zero-points int64 [tokens])."""
    obs = PerChannelMinMaxObserver(0)
    obs.update(x)
    scales, zps = obs.get_quant_params(num_bits, symmetric)
    s = torch.from_numpy(np.asarray(scales, np.float32)).reshape(-1, 1)
    z = torch.from_numpy(np.asarray(zps).astype(np.float32)).reshape(-1, 1)
    out, codes = fake_quantize_codes(x, s, z, num_bits, symmetric)
    return out, codes, np.asarray(scales, np.float32), np.asarray(zps, np.int64)
