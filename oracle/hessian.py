"""Hessian accumulation and damped Cholesky inverse (oracle; test infrastructure only).

Restates:
  * ``HessianAccumulator``        src/LLMCompressorSharp.TorchExtensions/Hessian/HessianAccumulator.cs:16-99
  * ``HessianInverseSolver``      src/LLMCompressorSharp.TorchExtensions/Hessian/HessianInverseSolver.cs:25-108
"""

from __future__ import annotations

import torch


class HessianAccumulator:
    """H = sum X^T X in fp32 over all Update calls (HessianAccumulator.cs:16-99).
    No 2/n normalisation: the reference accumulates the raw sum (:63-64)."""

    def __init__(self, in_features: int):
        if in_features <= 0:
            raise ValueError("inFeatures must be positive.")  # :28-31
        self.in_features = in_features
        self._h = torch.zeros(in_features, in_features, dtype=torch.float32)  # :34
        self.sample_count = 0

    def update(self, x: torch.Tensor) -> None:
        """HessianAccumulator.Update, :47-67."""
        if x.shape[-1] != self.in_features:  # :52-57
            raise ValueError(f"Input last dim ({x.shape[-1]}) must equal inFeatures ({self.in_features}).")
        flat = x.to(torch.float32).reshape(-1, self.in_features)  # :59-60
        self._h.add_(flat.t().matmul(flat))  # :63-64
        self.sample_count += flat.shape[0]  # :66

    def get_hessian(self) -> torch.Tensor:  # :71-75
        return self._h.detach().clone()

    def reset(self) -> None:  # :78-83
        self._h.zero_()
        self.sample_count = 0


def _cholesky_or_none(a: torch.Tensor):
    l, info = torch.linalg.cholesky_ex(a)
    return None if int(info) != 0 else l


def damped(h: torch.Tensor, damping_frac: float) -> torch.Tensor:
    """H' = H + f * mean(diag H) * I when f > 0 (HessianInverseSolver.cs:62-70)."""
    hw = h.detach().to(torch.float32).clone()
    if damping_frac > 0:
        diag_mean = hw.diagonal().mean().item()  # fp32 mean, read back as float (:64)
        lam = torch.tensor(damping_frac, dtype=torch.float32) * torch.tensor(diag_mean, dtype=torch.float32)
        hw.diagonal().add_(lam.item())  # :67-68
    return hw


def hessian_inverse(h: torch.Tensor, damping_frac: float) -> torch.Tensor:
    """HessianInverseSolver.Compute, :44-92.

    L = chol(H'); Linv = solve_triangular(L, I, upper=False); return Linv^T Linv.  On a
    Cholesky failure returns pinv(H') (:85-91)."""
    if h.dim() != 2 or h.shape[0] != h.shape[1]:
        raise ValueError(f"Hessian must be a square 2-D tensor; got shape {list(h.shape)}.")  # :48-53
    d = h.shape[0]
    hw = damped(h, damping_frac)
    low = _cholesky_or_none(hw)
    if low is None:
        return torch.linalg.pinv(hw)  # :90
    eye = torch.eye(d, dtype=torch.float32)
    linv = torch.linalg.solve_triangular(low, eye, upper=False)  # :80
    return linv.t().mm(linv)  # :83


def upper_factor(hinv: torch.Tensor) -> torch.Tensor:
    """U with U^T U = Hinv, i.e. chol(Hinv)^T; falls back to Hinv itself when that
    Cholesky fails (GptqBlockQuantizer.cs:105-118)."""
    hf = hinv.detach().to(torch.float32).contiguous()
    low = _cholesky_or_none(hf)
    if low is None:
        return hf.clone()
    return low.t().contiguous()
