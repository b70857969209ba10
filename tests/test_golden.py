"""Committed golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py).

CPU: the oracle still reproduces every fixture bit for bit.  GPU: the CUDA path, called
through the C ABI, against the fixtures (RTN bit-exact; GPTQ / SparseGPT within the stated
tolerances) without running the oracle."""

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
DEV = "cuda:0"


def load(name):
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as f:
        return {k: f[k] for k in f.files}


def rel_fro(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def test_oracle_reproduces_fixtures():
    sys.path.insert(0, GOLDEN)
    import make_golden

    for name, arrays in make_golden.cases().items():
        ref = load(name)
        assert sorted(ref) == sorted(arrays), name
        for k, v in arrays.items():
            assert np.array_equal(v, ref[k]), (name, k)


@pytest.mark.gpu
def test_hessian_matches_fixture():
    from llmcompressorsharp_b200 import HessianAccumulator

    g = load("hessian")
    acc = HessianAccumulator(200)
    acc.update(torch.from_numpy(g["x"]).to(torch.bfloat16).to(DEV))
    assert rel_fro(acc.get_hessian(), g["h"]) < 1e-5


@pytest.mark.gpu
def test_inverse_matches_fixture():
    from llmcompressorsharp_b200 import HessianInverseSolver

    g = load("inverse")
    h = torch.from_numpy(g["h"]).to(DEV)
    assert rel_fro(HessianInverseSolver.compute(h, 0.01), g["hinv"]) < 1e-4
    assert rel_fro(HessianInverseSolver.upper(h, 0.01), g["u"]) < 1e-4


@pytest.mark.gpu
def test_rtn_matches_fixture_bit_exact():
    from llmcompressorsharp_b200 import RtnConfig, rtn_quantize

    g = load("rtn_g128_asym4")
    w = torch.from_numpy(g["w"]).to(torch.bfloat16).to(DEV)
    deq, codes, scales, zps = rtn_quantize(w, RtnConfig(num_bits=4, symmetric=False, strategy="group", group_size=128))
    assert torch.equal(deq.float().cpu(), torch.from_numpy(g["deq"]))
    assert np.array_equal(scales.cpu().numpy(), g["scales"])
    assert np.array_equal(zps.cpu().numpy(), g["zps"].astype(np.int32))
    zp_e = np.repeat(g["zps"], 128, axis=1)
    nib = (g["codes"] - zp_e) & 0xF
    packed = ((nib[:, 0::2] << 4) | nib[:, 1::2]).astype(np.uint8)
    assert np.array_equal(codes.cpu().numpy(), packed)


@pytest.mark.gpu
def test_gptq_matches_fixture():
    from llmcompressorsharp_b200 import GPTQConfig, gptq_quantize_u

    g = load("gptq_g128_asym4")
    res = gptq_quantize_u(torch.from_numpy(g["w"]).to(DEV), torch.from_numpy(g["u"]).to(DEV),
                          GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128))
    assert np.array_equal(res.scales.cpu().numpy(), g["scales"])
    assert np.array_equal(res.zero_points.cpu().numpy(), g["zps"].astype(np.int32))
    assert (res.wq.cpu().numpy() == g["wq"]).mean() >= 0.999
    h = torch.from_numpy(g["h"]).double()
    w = torch.from_numpy(g["w"]).double()

    def err(wq):
        dw = w - torch.as_tensor(wq).double().cpu()
        return float(torch.einsum("ij,jk,ik->", dw, h, dw))

    assert abs(err(res.wq) / err(g["wq"]) - 1) < 0.01


@pytest.mark.gpu
def test_sparsegpt_matches_fixture():
    from llmcompressorsharp_b200 import SparseGPTConfig, sparsegpt_prune_u

    g = load("sparsegpt_2_4")
    out, mask = sparsegpt_prune_u(torch.from_numpy(g["w"]).to(DEV), torch.from_numpy(g["u"]).to(DEV),
                                  SparseGPTConfig(sparsity=0.5, mask_structure="2:4"))
    assert (mask.cpu().numpy().astype(bool) == g["mask"]).mean() >= 0.999
    assert rel_fro(out, g["out"]) < 1e-3


@pytest.mark.gpu
def test_pinv_fallback_matches_fixture():
    """HessianInverseSolver.cs:85-91: a dead input channel and no damping leave no Cholesky
    factor; the pseudo-inverse agrees with the oracle's torch.linalg.pinv to 1e-3 (an fp32
    eigensolver against an fp32 SVD).  The dead channel's row and column are exactly zero (the
    oracle's SVD leaves residue near 1e-9 of the largest entry there), so GPTQ's factor falls
    back to Hinv (GptqBlockQuantizer.cs:112-118), as the oracle's does."""
    from llmcompressorsharp_b200 import HessianInverseSolver

    g = load("pinv_dead_channel")
    h = torch.from_numpy(g["h"]).to(DEV)
    hinv = HessianInverseSolver.compute(h, 0.0)
    assert rel_fro(hinv, g["hinv"]) < 1e-3
    assert torch.count_nonzero(hinv[11]) == 0 and torch.count_nonzero(hinv[:, 11]) == 0
    u = HessianInverseSolver.upper(h, 0.0)
    assert np.array_equal(g["u"], g["hinv"])
    assert torch.equal(u, hinv)
    assert rel_fro(u, g["u"]) < 1e-3


@pytest.mark.gpu
def test_act_order_gptq_matches_fixture():
    from llmcompressorsharp_b200 import GPTQConfig, gptq_quantize_act_order

    g = load("gptq_act_order_g64")
    res, perm = gptq_quantize_act_order(torch.from_numpy(g["w"]).to(torch.bfloat16).to(DEV), torch.from_numpy(g["h"]).to(DEV),
                                        GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=64,
                                                   dampening_frac=0.01))
    assert np.array_equal(perm.cpu().numpy().astype(np.int64), g["perm"])
    assert np.array_equal(res.scales.cpu().numpy(), g["scales"])
    assert np.array_equal(res.zero_points.cpu().numpy(), g["zps"].astype(np.int32))
    assert (res.wq.cpu().numpy() == g["wq"]).mean() >= 0.999


@pytest.mark.gpu
def test_per_token_matches_fixture_bit_exact():
    from llmcompressorsharp_b200 import quantize_per_token

    g = load("per_token_int8_sym")
    codes, scales, zps, deq = quantize_per_token(torch.from_numpy(g["x"]).to(torch.bfloat16).to(DEV), 8, True,
                                                 want_values=True)
    assert np.array_equal(scales.cpu().numpy(), g["scales"])
    assert np.array_equal(zps.cpu().numpy(), g["zps"].astype(np.int32))
    assert np.array_equal(codes.cpu().to(torch.int64).numpy(), g["codes"].astype(np.int64))
    assert np.array_equal(deq.float().cpu().numpy(), g["deq"])


@pytest.mark.gpu
def test_smoothquant_matches_fixture_bit_exact():
    from llmcompressorsharp_b200.smoothquant import smooth_apply

    g = load("smoothquant_a05")
    sw, bw, s = smooth_apply(torch.from_numpy(g["smooth"]).to(torch.bfloat16).to(DEV),
                             torch.from_numpy(g["balance"]).to(torch.bfloat16).to(DEV),
                             torch.from_numpy(g["act_max"]).to(DEV), 0.5)
    assert np.array_equal(s.cpu().numpy(), g["s"])
    assert np.array_equal(sw.float().cpu().numpy(), g["new_smooth"])
    assert np.array_equal(bw.float().cpu().numpy(), g["new_balance"])


@pytest.mark.gpu
def test_awq_search_matches_fixture():
    from llmcompressorsharp_b200 import RtnConfig, awq_search

    g = load("awq_g128")
    s, k, mse = awq_search(torch.from_numpy(g["w"]).to(torch.bfloat16).to(DEV), torch.from_numpy(g["act_max"]).to(DEV),
                           20, RtnConfig(4, False, "group", group_size=128))
    rmse, rk = g["mse"], int(g["k"])
    assert np.allclose(mse.cpu().numpy(), rmse, rtol=1e-4)
    assert k == rk or abs(rmse[k - 1] / rmse[rk - 1] - 1) < 1e-4
    if k == rk:
        assert rel_fro(s, g["s"]) < 1e-6
