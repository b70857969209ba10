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
