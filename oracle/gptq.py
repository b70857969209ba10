"""GPTQ column-block solve (oracle; test infrastructure only).

Restates ``GptqBlockQuantizer.Quantize`` (src/LLMCompressorSharp.Core/Algorithms/Gptq/
GptqBlockQuantizer.cs:71-190), ``ComputeScaleZeroPoint`` (:196-234) and
``FakeQuantizeColumn`` (:240-274), plus the group strategy extension (one MinMax
observer per (row, group), computed before the loop from the ORIGINAL weight, the
same rule ComputeScaleZeroPoint applies per row; parity unpinned).

The per-row scalar FakeQuantize calls of the reference (:259-263) are element-wise, so
a per-row scale broadcast over the column gives identical values.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .affine import compute_affine_params, affine_params_array, group_minmax, observer_fold
from .fakequant import fake_quantize_codes
from .hessian import hessian_inverse, upper_factor

NUMERIC_EPSILON = np.float32(1e-10)  # GptqBlockQuantizer.cs:48


@dataclass
class GPTQConfig:
    """GPTQConfig.cs:22-59 (defaults kept) plus ``group_size`` for strategy 'group'."""

    num_bits: int = 4
    symmetric: bool = True
    strategy: str = "channel"  # 'tensor' | 'channel' | 'group'
    channel_axis: int = 0
    block_size: int = 128
    dampening_frac: float = 0.01
    act_order: bool = False
    group_size: int = 128


def compute_scale_zero_point(w: torch.Tensor, cfg: GPTQConfig):
    """ComputeScaleZeroPoint, :196-234.  Returns (scales, zps) shaped for broadcasting
    as [m, G] where G = 1 (tensor/channel) or the group count."""
    m, n = w.shape
    wf = w.detach().to(torch.float32)
    # One new MinMaxObserver per tensor / row (:200-203, :212-222): observer_fold.
    if cfg.strategy == "tensor":
        mn, mx = observer_fold(wf.min().item(), wf.max().item())
        s, z = compute_affine_params(float(mn), float(mx), cfg.num_bits, cfg.symmetric)
        return (np.full((m, 1), s, dtype=np.float32), np.full((m, 1), z, dtype=np.int64))
    if cfg.strategy == "channel":
        if cfg.channel_axis != 0:
            raise NotImplementedError("per-channel GPTQ uses output channels (axis 0)")
        mn, mx = observer_fold(wf.amin(dim=1).numpy(), wf.amax(dim=1).numpy())
        s, z = affine_params_array(mn, mx, cfg.num_bits, cfg.symmetric)
        return s.reshape(m, 1), z.reshape(m, 1)
    if cfg.strategy == "group":
        mins, maxs = group_minmax(wf, cfg.group_size)
        mn, mx = observer_fold(mins.numpy(), maxs.numpy())
        s, z = affine_params_array(mn, mx, cfg.num_bits, cfg.symmetric)
        return s, z
    raise NotImplementedError(f"Quantization strategy '{cfg.strategy}' is not supported by GptqBlockQuantizer.")


def _column_params(scales, zps, cfg: GPTQConfig, j: int):
    g = 0 if scales.shape[1] == 1 else j // cfg.group_size
    return (torch.from_numpy(np.ascontiguousarray(scales[:, g])),
            torch.from_numpy(np.ascontiguousarray(zps[:, g]).astype(np.float32)))


def gptq_quantize_u(weight: torch.Tensor, upper: torch.Tensor, cfg: GPTQConfig):
    """The column loop of Quantize (:122-181) given the factor U.

    Returns (wq fp32 [m,n], codes int32 [m,n], scales [m,G] fp32, zps [m,G] int64)."""
    if cfg.act_order:
        raise NotImplementedError("GPTQConfig.ActOrder=true is not yet implemented.")  # :77-82
    scales, zps = compute_scale_zero_point(weight, cfg)  # :97
    return _column_loop(weight.detach().to(torch.float32).clone(), upper, cfg, scales, zps, None)


def act_order_perm(h: torch.Tensor) -> torch.Tensor:
    """Extension (parity unpinned; the reference rejects ActOrder, GPTQModifier.cs:47-56): the
    GPTQ activation order, columns by decreasing Hessian diagonal.  Stable: equal values keep
    index order; NaN entries come first."""
    diag = torch.diagonal(h).to(torch.float32).tolist()
    order = sorted(range(len(diag)), key=lambda i: (0 if diag[i] != diag[i] else 1,
                                                    0.0 if diag[i] != diag[i] else -diag[i], i))
    return torch.tensor(order, dtype=torch.int64)


def gptq_quantize_act_order(weight: torch.Tensor, h: torch.Tensor, damping_frac: float, cfg: GPTQConfig):
    """Extension (parity unpinned): GPTQ with activation order and static groups.

    perm = act_order_perm(H); U_p is the factor of H[perm][:, perm] (hessian_inverse and
    upper_factor as for any Hessian); scales and zero-points come from the ORIGINAL weight per
    original column group, before the loop, as ComputeScaleZeroPoint does (:97); the loop of
    Quantize (:122-181) runs over W[:, perm] against U_p, column a quantised with the parameters
    of original column perm[a]; results are scattered back to the original columns.
    Returns (wq fp32 [m,n], codes int32 [m,n], scales, zps, perm)."""
    perm = act_order_perm(h)
    hp = h.detach().to(torch.float32)[perm][:, perm].contiguous()
    up = upper_factor(hessian_inverse(hp, damping_frac))
    scales, zps = compute_scale_zero_point(weight, cfg)
    wp = weight.detach().to(torch.float32)[:, perm].clone()
    wq_p, codes_p, _, _ = _column_loop(wp, up, cfg, scales, zps, perm)
    wq = torch.empty_like(wq_p)
    codes = torch.empty_like(codes_p)
    wq[:, perm] = wq_p
    codes[:, perm] = codes_p
    return wq, codes, scales, zps, perm


def _column_loop(w_work: torch.Tensor, upper: torch.Tensor, cfg: GPTQConfig, scales, zps, col_of):
    """The block loop of Quantize, :122-181, on the fp32 working copy w_work (modified in place).
    Column aj takes the parameters of column col_of[aj] (aj itself when col_of is None)."""
    m, n = w_work.shape
    bs = cfg.block_size
    wq = torch.zeros_like(w_work)  # :92
    codes = torch.zeros(m, n, dtype=torch.int32)
    u = upper.detach().to(torch.float32)
    for i1 in range(0, n, bs):  # :124
        i2 = min(i1 + bs, n)
        cnt = i2 - i1
        err1 = torch.zeros(m, cnt, dtype=torch.float32)  # :131
        for j in range(cnt):  # :134
            aj = i1 + j
            w_col = w_work[:, aj].clone()  # :141
            s, z = _column_params(scales, zps, cfg, aj if col_of is None else int(col_of[aj]))
            q, c = fake_quantize_codes(w_col, s, z, cfg.num_bits, cfg.symmetric)  # :142
            wq[:, aj] = q  # :143
            codes[:, aj] = c
            pivot = np.float32(u[aj, aj].item())  # :146
            if abs(pivot) < NUMERIC_EPSILON:  # :147-150
                continue
            err = (w_col - q).div(float(pivot))  # :153
            err1[:, j] = err  # :156
            rem = cnt - j - 1
            if rem > 0:  # :160-168
                u_row = u[aj, aj + 1:i2]
                w_work[:, aj + 1:i2].sub_(err.unsqueeze(1).mm(u_row.unsqueeze(0)))
        tail = n - i2
        if tail > 0:  # :173-180
            w_work[:, i2:].sub_(err1.mm(u[i1:i2, i2:]))
    return wq, codes, scales, zps


def gptq_quantize(weight: torch.Tensor, hinv: torch.Tensor, cfg: GPTQConfig):
    """GptqBlockQuantizer.Quantize(W, Hinv, cfg), :71-190: U = chol(Hinv)^T with the
    Hinv fallback, then the column loop."""
    return gptq_quantize_u(weight, upper_factor(hinv), cfg)


def reconstruction_error(w: torch.Tensor, wq: torch.Tensor, h: torch.Tensor) -> float:
    """||W X^T - Wq X^T||_F^2 over the calibration set = tr(dW H dW^T) with H = sum X^T X,
    computed in fp64."""
    dw = (w.to(torch.float64) - wq.to(torch.float64))
    return float(torch.einsum("ij,jk,ik->", dw, h.to(torch.float64), dw))
