"""SparseGPT column-block pruning (oracle; test infrastructure only; parity unpinned).

The reference has SparseGPT only as a plan:
docs/superpowers/plans/2026-05-18-phase-4c-sparsegpt.md:37-59 (algorithm, per-row mask
rule) and :1584-1656 (block loop).  The plan's loop uses full-Hinv entries, the same
inconsistency GptqBlockQuantizer.cs:37-44 documents and corrects for GPTQ; this oracle
uses the corrected U-factor form of the GPTQ loop (GptqBlockQuantizer.cs:124-181), with
the mask-selection step in place of fake-quantisation:

  per block [i1, i2): saliency = W_blk^2 / diag(U_blk)^2 taken from the block's
  snapshot (plan :1598-1602, with the U diagonal); the per-row mask keeps the top
  entries: unstructured keeps ceil((1 - sparsity) * cnt) per row in the block, N:M keeps
  the N largest of each M consecutive columns (plan :37-59; algorithm-mapping.md:200-212);
  then for each column j: q = w * keep, err = (w - q) / U[j,j], in-block rank-1 update
  and the tail update as in GPTQ.

Ties in saliency are broken towards the lower column index (stable sort order).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .gptq import NUMERIC_EPSILON


def select_mask(sal: torch.Tensor, sparsity: float, mask_n: int, mask_m: int) -> torch.Tensor:
    """Per-row keep mask for a block's saliency [m, cnt].  N:M when mask_m > 0."""
    m, cnt = sal.shape
    keep = torch.zeros(m, cnt, dtype=torch.bool)
    if mask_m > 0:
        for g0 in range(0, cnt, mask_m):
            g = sal[:, g0:g0 + mask_m]
            # stable descending order: larger saliency first, lower index on ties
            order = torch.sort(-g, dim=1, stable=True).indices[:, :mask_n]
            keep[:, g0:g0 + mask_m].scatter_(1, order, True)
        return keep
    n_keep = int(math.ceil((1.0 - sparsity) * cnt - 1e-9))
    order = torch.sort(-sal, dim=1, stable=True).indices[:, :n_keep]
    keep.scatter_(1, order, True)
    return keep


def sparsegpt_prune_u(weight: torch.Tensor, upper: torch.Tensor, block_size: int = 128,
                      sparsity: float = 0.5, mask_n: int = 0, mask_m: int = 0):
    """Returns (pruned fp32 weight [m,n], keep mask bool [m,n])."""
    m, n = weight.shape
    w = weight.detach().to(torch.float32).clone()
    u = upper.detach().to(torch.float32)
    out = torch.zeros_like(w)
    mask = torch.zeros(m, n, dtype=torch.bool)
    for i1 in range(0, n, block_size):
        i2 = min(i1 + block_size, n)
        cnt = i2 - i1
        d = u[i1:i2, i1:i2].diagonal()
        sal = w[:, i1:i2].pow(2) / d.pow(2).clamp_min(1e-10).unsqueeze(0)
        keep = select_mask(sal, sparsity, mask_n, mask_m)
        mask[:, i1:i2] = keep
        err1 = torch.zeros(m, cnt)
        for j in range(cnt):
            aj = i1 + j
            col = w[:, aj].clone()
            q = torch.where(keep[:, j], col, torch.zeros_like(col))
            out[:, aj] = q
            piv = np.float32(u[aj, aj].item())
            if abs(piv) < NUMERIC_EPSILON:
                continue
            err = (col - q).div(float(piv))
            err1[:, j] = err
            if j + 1 < cnt:
                w[:, aj + 1:i2].sub_(err.unsqueeze(1).mm(u[aj, aj + 1:i2].unsqueeze(0)))
        if i2 < n:
            w[:, i2:].sub_(err1.mm(u[i1:i2, i2:]))
    return out, mask
