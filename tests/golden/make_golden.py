"""Generates the committed golden fixtures (tests/golden/*.npz) from the oracle.

The reference (C# on TorchSharp) cannot run in this environment, so these vectors are the
oracle's outputs on small seeded inputs; the oracle itself is pinned to the reference's own
known-answer tests (tests/test_oracle_kats.py).  The fixtures freeze those outputs: the CPU
suite checks that the oracle still reproduces them, and the GPU suite checks the CUDA path
against them without running the oracle.

    python tests/golden/make_golden.py      # rewrites tests/golden/*.npz
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import gptq as o_gptq, hessian as o_hess, rtn as o_rtn, sparsegpt as o_sp  # noqa: E402


def gen(seed):
    return torch.Generator().manual_seed(seed)


def cases():
    out = {}
    # Hessian of bf16 activations (exact products, fp32 sums), 300 x 200
    x = torch.randn(300, 200, generator=gen(1)).to(torch.bfloat16)
    acc = o_hess.HessianAccumulator(200)
    acc.update(x)
    out["hessian"] = {"x": x.float().numpy(), "h": acc.get_hessian().numpy()}
    # damped inverse and upper factor, d = 160
    a = torch.randn(400, 160, generator=gen(2))
    h = a.t() @ a
    hinv = o_hess.hessian_inverse(h, 0.01)
    out["inverse"] = {"h": h.numpy(), "hinv": hinv.numpy(), "u": o_hess.upper_factor(hinv).numpy()}
    # RTN asym int4 g128 on bf16 with outliers, 48 x 512
    w = torch.randn(48, 512, generator=gen(3)) * 0.02
    w = torch.where(torch.rand(48, 512, generator=gen(4)) < 0.01, w * 20, w).to(torch.bfloat16)
    deq, codes, s, z = o_rtn.rtn_quantize(w, o_rtn.RtnConfig(4, False, "group", group_size=128))
    out["rtn_g128_asym4"] = {"w": w.float().numpy(), "deq": deq.float().numpy(), "codes": codes.numpy(),
                             "scales": np.asarray(s, np.float32), "zps": np.asarray(z, np.int64)}
    # GPTQ asym int4 g128 on a 64 x 256 fp32 weight
    xg = torch.randn(1024, 256, generator=gen(5))
    hg = xg.t() @ xg
    wg = torch.randn(64, 256, generator=gen(6)) * 0.02
    ug = o_hess.upper_factor(o_hess.hessian_inverse(hg, 0.01))
    cfg = o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128)
    wq, cg, sg, zg = o_gptq.gptq_quantize_u(wg, ug, cfg)
    out["gptq_g128_asym4"] = {"w": wg.numpy(), "u": ug.numpy(), "h": hg.numpy(), "wq": wq.numpy(), "codes": cg.numpy(),
                              "scales": np.asarray(sg, np.float32), "zps": np.asarray(zg, np.int64)}
    # SparseGPT 2:4 on the same weight and factor
    ps, pm = o_sp.sparsegpt_prune_u(wg, ug, 128, 0.5, 2, 4)
    out["sparsegpt_2_4"] = {"w": wg.numpy(), "u": ug.numpy(), "out": ps.numpy(), "mask": pm.numpy()}
    return out


def main():
    for name, arrays in cases().items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        print(name, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
