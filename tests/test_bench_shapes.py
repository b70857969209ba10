"""Parity at the shapes the Llama-3-8B GPTQ job runs, on the path that job takes.

  * down_proj: a d = 14,336 Hessian from one 65,536-row bf16 update call (the job's update
    size, the pair kernel with its token splits), the factor U = chol(H'^-1)^T through
    llmc_chol_inverse(want_upper = 1) (HessianInverseSolver.cs:44-92 and
    GptqBlockQuantizer.cs:105-118), and the GPTQ solve of a 256-row down_proj slice
    (GptqBlockQuantizer.cs:71-190) over all 14,336 columns.
  * gate/up: the MLP-input site (d = 4,096) with both 14,336 x 4,096 weights solved as one
    stacked 28,672-row matrix by GptqPipeline.solve_site, whose far-tail GEMMs are the job's
    largest (M = 28,672).

The oracle computes every stage from its own results (H, Hinv, U, the column loop) on the CPU.
Bars: H within 1e-5 relative Frobenius, U within 1e-4; GPTQ scales and zero-points equal,
fake-quantised values equal on >= 99.9 % of elements, tr(dW H dW^T) within 1 %.
Activations have per-channel scales exp(N(0, 0.5^2)) so that H is not a multiple of I."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import gptq as o_gptq, hessian as o_hess

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
T = 65536
CFG = dict(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128)


def rel_fro(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm())


def activations(rows, d, seed):
    g = torch.Generator(DEV).manual_seed(seed)
    scale = torch.exp(0.5 * torch.randn(d, device=DEV, generator=g))
    return (torch.randn(rows, d, device=DEV, generator=g) * scale).to(torch.bfloat16)


def oracle_hessian(x_dev, d):
    ref = o_hess.HessianAccumulator(d)
    for r0 in range(0, x_dev.shape[0], 8192):
        ref.update(x_dev[r0:r0 + 8192].cpu())
    return ref.get_hessian()


def gptq_bars(w, wq_dev, scales_dev, zps_dev, wq_ref, s_ref, z_ref, h):
    assert np.array_equal(scales_dev.cpu().numpy().reshape(-1), np.asarray(s_ref, np.float32).reshape(-1))
    assert np.array_equal(zps_dev.cpu().numpy().reshape(-1), np.asarray(z_ref).reshape(-1))
    agree = (wq_dev.cpu() == wq_ref).float().mean().item()
    assert agree >= 0.999, agree
    e_dev = o_gptq.reconstruction_error(w, wq_dev.cpu(), h)
    e_ref = o_gptq.reconstruction_error(w, wq_ref, h)
    assert abs(e_dev / e_ref - 1) < 0.01, (e_dev, e_ref)


def test_down_proj_chain_at_d14336():
    from llmcompressorsharp_b200 import GPTQConfig, HessianAccumulator, HessianInverseSolver, gptq_quantize_u

    d, m = 14336, 256
    x = activations(T, d, 14336)
    acc = HessianAccumulator(d, DEV)
    acc.update(x)  # one 65,536-row call, as the job makes
    h_dev = acc.get_hessian()
    h_ref = oracle_hessian(x, d)
    del x
    assert rel_fro(h_dev, h_ref) < 1e-5

    u_dev = HessianInverseSolver.upper(acc.raw(), 0.01, upper_only=True)
    acc.dispose()
    hinv_ref = o_hess.hessian_inverse(h_ref, 0.01)
    u_ref = o_hess.upper_factor(hinv_ref)
    del hinv_ref
    assert rel_fro(u_dev, u_ref) < 1e-4
    assert torch.count_nonzero(torch.tril(u_dev, -1)) == 0

    w = (torch.randn(m, d, generator=torch.Generator().manual_seed(5)) * 0.02).to(torch.bfloat16)
    res = gptq_quantize_u(w.to(DEV), u_dev, GPTQConfig(**CFG))
    wq_r, _, s_r, z_r = o_gptq.gptq_quantize_u(w, u_ref, o_gptq.GPTQConfig(**CFG))
    gptq_bars(w, res.wq, res.scales, res.zero_points, wq_r, s_r, z_r, h_ref)


def test_gate_up_stack_at_m28672():
    from llmcompressorsharp_b200.gptq import GPTQConfig
    from llmcompressorsharp_b200.pipeline import GptqPipeline, SiteSpec

    d, m = 4096, 14336
    site = SiteSpec("mlp_in", d, [("gate_proj", m), ("up_proj", m)])
    pipe = GptqPipeline([site], GPTQConfig(dampening_frac=0.01, **CFG), torch.device(DEV), chunk_rows=T,
                        keep_wq=True)
    try:
        x = activations(T, d, 4096)
        g = torch.Generator().manual_seed(7)
        w_cpu = {n: (torch.randn(m, d, generator=g) * 0.02).to(torch.bfloat16) for n in ("gate_proj", "up_proj")}
        weights = {n: t.to(DEV) for n, t in w_cpu.items()}
        outputs = pipe.alloc_outputs(weights)
        pipe.accumulate(site, x)
        pipe.solve_site(site, pipe.hessian_ptr(site.name), weights, outputs)
        torch.cuda.synchronize()
        h_ref = oracle_hessian(x, d)
        del x
        u_ref = o_hess.upper_factor(o_hess.hessian_inverse(h_ref, 0.01))
        for name in ("gate_proj", "up_proj"):
            out = outputs[name]
            wq_r, _, s_r, z_r = o_gptq.gptq_quantize_u(w_cpu[name], u_ref, o_gptq.GPTQConfig(**CFG))
            gptq_bars(w_cpu[name], out["wq"], out["scales"], out["zero_points"], wq_r, s_r, z_r, h_ref)
    finally:
        pipe.close()


def test_factor_at_d28672_against_fp64():
    """Llama-3-70B's widest site (down_proj input, d = 28,672): the Hessian of 32,768 bf16 rows
    (fewer rows than columns, so H' is only as well conditioned as the damping makes it) and
    U = chol(H'^-1)^T from llmc_chol_inverse(want_upper = 1), against the same chain of
    HessianInverseSolver.cs:44-92 / GptqBlockQuantizer.cs:105-118 in fp64 on the device
    (torch.linalg, used here only as the checker: the CPU oracle's fp32 chain takes too long at
    this width).  H' is the oracle's damping of the device's H.  Bar: U within 1e-4 relative
    Frobenius on a sample of 256 rows, and nothing below the diagonal."""
    from llmcompressorsharp_b200 import HessianAccumulator, HessianInverseSolver

    d = 28672
    x = activations(32768, d, 28672)
    acc = HessianAccumulator(d, DEV)
    acc.update(x)
    del x
    u_dev = HessianInverseSolver.upper(acc.raw(), 0.01, upper_only=True)
    h = acc.get_hessian()
    acc.dispose()
    hd = o_hess.damped(h, 0.01).double()
    del h
    low = torch.linalg.cholesky(hd)
    del hd
    hinv = torch.cholesky_inverse(low)
    del low
    u_ref = torch.linalg.cholesky(hinv, upper=True)
    del hinv
    rows = torch.randperm(d, generator=torch.Generator().manual_seed(3))[:256].to(DEV)
    assert rel_fro(u_dev[rows], u_ref[rows]) < 1e-4
    assert torch.count_nonzero(torch.tril(u_dev, -1)) == 0
