"""GPTQ activation order (extension; the reference rejects ActOrder, GPTQModifier.cs:47-56):
the CUDA path against the oracle's restatement (oracle/gptq.py gptq_quantize_act_order).

Bars as for GPTQ: the permutation and the permuted Hessian exact; scales and zero-points equal;
fake-quantised values equal on >= 99.9 % of elements; packed codes equal where the values are;
tr(dW H dW^T) within 1 % of the oracle's.  Parity unpinned (no reference code)."""

import numpy as np
import pytest
import torch

from oracle import fakequant as o_fq, gptq as o_gptq, hessian as o_hess

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def hessian(d, rows, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, d, generator=g) * torch.exp(torch.randn(d, generator=g))
    return x.t() @ x


def test_perm_is_stable_descending_with_nan_first():
    from llmcompressorsharp_b200 import act_order_perm

    diag = torch.tensor([1.0, 5.0, 5.0, float("nan"), 0.0, 7.0, 5.0, float("nan"), -1.0])
    h = torch.diag(diag)
    got = act_order_perm(h.to(DEV)).cpu().to(torch.int64)
    assert got.tolist() == o_gptq.act_order_perm(h).tolist() == [3, 7, 5, 1, 2, 6, 0, 4, 8]


@pytest.mark.parametrize("d", [64, 1000, 4096])
def test_perm_and_permuted_hessian_match_oracle(d):
    import ctypes as C

    from llmcompressorsharp_b200 import _lib, act_order_perm

    h = hessian(d, 2 * d, d)
    perm = act_order_perm(h.to(DEV))
    ref = o_gptq.act_order_perm(h)
    assert torch.equal(perm.cpu().to(torch.int64), ref)
    for upper_only in (0, 1):
        src = torch.triu(h) + torch.tril(torch.full_like(h, 9.0), -1) if upper_only else h
        hd = src.to(DEV)
        out = torch.empty(d, d, device=DEV)
        _lib.call("llmc_permute_hessian", C.c_void_p(_lib.ctx_for(0)), _lib.ptr(hd), C.c_int64(d), C.c_int64(d),
                  C.c_int32(upper_only), _lib.ptr(perm), _lib.ptr(out), C.c_int64(d))
        assert torch.equal(out.cpu(), h[ref][:, ref])


@pytest.mark.parametrize("strategy,sym,bits,gs", [("group", False, 4, 128), ("group", True, 4, 64),
                                                  ("channel", False, 4, 128), ("tensor", True, 8, 128),
                                                  ("group", False, 8, 128)])
@pytest.mark.parametrize("m,n", [(192, 512), (70, 384)])
def test_act_order_gptq_matches_oracle(strategy, sym, bits, gs, m, n):
    from llmcompressorsharp_b200 import GPTQConfig, gptq_quantize_act_order

    h = hessian(n, 4 * n, m + n)
    w = (torch.randn(m, n, generator=torch.Generator().manual_seed(n)) * 0.02).to(torch.bfloat16)
    cfg = dict(num_bits=bits, symmetric=sym, strategy=strategy, group_size=gs, block_size=128)
    res, perm = gptq_quantize_act_order(w.to(DEV), h.to(DEV), GPTQConfig(dampening_frac=0.01, **cfg))
    wq_r, codes_r, s_r, z_r, perm_r = o_gptq.gptq_quantize_act_order(w, h, 0.01, o_gptq.GPTQConfig(**cfg))
    assert torch.equal(perm.cpu().to(torch.int64), perm_r)
    k = 1 if strategy == "tensor" else None
    assert np.array_equal(res.scales.cpu().numpy().reshape(-1)[:k], np.asarray(s_r, np.float32).reshape(-1)[:k])
    assert np.array_equal(res.zero_points.cpu().numpy().reshape(-1)[:k], np.asarray(z_r).reshape(-1)[:k])
    same = res.wq.cpu() == wq_r
    assert same.float().mean().item() >= 0.999
    if bits <= 4:
        zp_e = torch.from_numpy(np.asarray(z_r))
        if zp_e.dim() == 2 and zp_e.shape[1] > 1:
            zp_e = zp_e[:, torch.arange(n) // gs]
        elif zp_e.numel() == 1:
            zp_e = zp_e.reshape(1, 1).expand(m, 1)
        ref_packed = o_fq.pack_int4_rows(codes_r, zp_e)
        got = res.codes.cpu()
        rows_same = same.all(dim=1)
        assert torch.equal(got[rows_same], ref_packed[rows_same])
    else:
        rows_same = same.all(dim=1)
        assert torch.equal(res.codes.cpu()[rows_same], codes_r.to(torch.uint8)[rows_same])
    e_dev = o_gptq.reconstruction_error(w, res.wq.cpu(), h)
    e_ref = o_gptq.reconstruction_error(w, wq_r, h)
    assert abs(e_dev / e_ref - 1) < 0.01, (e_dev, e_ref)


def test_act_order_with_sorted_diagonal_equals_plain_gptq():
    """When diag(H) is already decreasing, the order is the identity and the result is plain GPTQ."""
    from llmcompressorsharp_b200 import GPTQConfig, HessianInverseSolver, gptq_quantize_act_order, gptq_quantize_u

    n, m = 256, 128
    g = torch.Generator().manual_seed(2)
    a = torch.randn(n, n, generator=g) * 0.01
    h = torch.diag(torch.linspace(50.0, 1.0, n)) + a @ a.t()
    w = (torch.randn(m, n, generator=g) * 0.02).to(torch.bfloat16)
    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, dampening_frac=0.01)
    res, perm = gptq_quantize_act_order(w.to(DEV), h.to(DEV), cfg)
    assert torch.equal(perm.cpu(), torch.arange(n, dtype=torch.int32))
    plain = gptq_quantize_u(w.to(DEV), HessianInverseSolver.upper(h.to(DEV), 0.01), cfg)
    assert torch.equal(res.wq, plain.wq) and torch.equal(res.codes, plain.codes)
    assert torch.equal(res.scales, plain.scales) and torch.equal(res.zero_points, plain.zero_points)


def test_reference_entry_points_still_reject_act_order():
    """GptqBlockQuantizer.Quantize and llmc_gptq_quantize keep the reference's NotSupported
    (GptqBlockQuantizer.cs:77-82, GPTQModifierTests.cs:130-141)."""
    from llmcompressorsharp_b200 import GPTQConfig, GptqBlockQuantizer, NotSupportedError

    with pytest.raises(NotSupportedError, match="ActOrder"):
        GptqBlockQuantizer.quantize(torch.ones(2, 2, device=DEV), torch.eye(2, device=DEV), GPTQConfig(act_order=True))
