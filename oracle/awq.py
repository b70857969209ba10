"""AWQ grid search of per-input-channel scales (oracle; test infrastructure only;
parity unpinned).

The reference has AWQ as a design sketch only: docs/llmcompressorsharp/algorithm-mapping.md:214-249.
For k = 1..nGrid: alpha = k/nGrid; s = actMax^alpha / wMax^(1-alpha) clamped >= 1e-4;
mse = mean((FQ(W * s) / s - W)^2); keep the s with the lowest mse (first on ties).
FQ here is the group-wise RTN of the weight (strategy given by the config), the same
observer + fake-quant chain as RTN.
"""

from __future__ import annotations

import numpy as np
import torch

from .rtn import RtnConfig, rtn_quantize


def awq_search(weight: torch.Tensor, act_max: np.ndarray, n_grid: int, cfg: RtnConfig):
    """Returns (best scale [n] fp32, best alpha index k, per-k mse list)."""
    w = weight.detach().to(torch.float32)
    a = torch.from_numpy(np.asarray(act_max, np.float32))
    wmax = w.abs().amax(dim=0)
    best_mse = np.inf
    best_s = None
    best_k = 0
    mses = []
    for k in range(1, n_grid + 1):
        alpha = np.float32(k) / np.float32(n_grid)
        s = (a.pow(float(alpha)) / wmax.pow(float(np.float32(1) - alpha))).clamp(min=1e-4)
        ws = w * s.unsqueeze(0)
        fq, _, _, _ = rtn_quantize(ws, cfg)
        back = fq.to(torch.float32) / s.unsqueeze(0)
        mse = float((back - w).pow(2).mean().item())
        mses.append(mse)
        if mse < best_mse:
            best_mse, best_s, best_k = mse, s.clone(), k
    return best_s, best_k, mses
