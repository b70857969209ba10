"""Generates the committed golden fixtures (tests/golden/*.npz) from the oracle.

The reference (C# on TorchSharp) cannot run in this environment, so these vectors are the
oracle's outputs on small seeded inputs; the oracle itself is pinned to the reference's own
known-answer tests (tests/test_oracle_kats.py).  The fixtures freeze those outputs: the CPU
suite checks that the oracle still reproduces them, and the GPU suite checks the CUDA path
against them without running the oracle.

    python tests/golden/make_golden.py [name ...]   # rewrites tests/golden/*.npz (or those named)
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import awq as o_awq, gptq as o_gptq, hessian as o_hess, pertoken as o_pt, rtn as o_rtn  # noqa: E402
from oracle import smoothquant as o_sq, sparsegpt as o_sp  # noqa: E402


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
    # the pinv fallback: an undamped Hessian with a dead input channel, d = 96
    xs = torch.randn(400, 96, generator=gen(7))
    xs[:, 11] = 0.0
    hs = xs.t() @ xs
    hinv_s = o_hess.hessian_inverse(hs, 0.0)
    out["pinv_dead_channel"] = {"h": hs.numpy(), "hinv": hinv_s.numpy(), "u": o_hess.upper_factor(hinv_s).numpy()}
    # GPTQ with activation order and static groups (asym int4 g64) on a 48 x 192 bf16 weight
    xa = torch.randn(768, 192, generator=gen(8)) * torch.exp(0.5 * torch.randn(192, generator=gen(9)))
    ha = xa.t() @ xa
    wa = (torch.randn(48, 192, generator=gen(10)) * 0.02).to(torch.bfloat16)
    acfg = o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=64, block_size=128)
    wq_a, c_a, s_a, z_a, p_a = o_gptq.gptq_quantize_act_order(wa, ha, 0.01, acfg)
    out["gptq_act_order_g64"] = {"w": wa.float().numpy(), "h": ha.numpy(), "wq": wq_a.numpy(), "codes": c_a.numpy(),
                                 "scales": np.asarray(s_a, np.float32), "zps": np.asarray(z_a, np.int64),
                                 "perm": p_a.numpy()}
    # per-token int8 (symmetric) of bf16 activations with outlier channels and an all-zero row
    xt = torch.randn(96, 640, generator=gen(11)) * torch.where(torch.rand(640, generator=gen(12)) < 0.02, 40.0, 1.0)
    xt[5] = 0.0
    xt = xt.to(torch.bfloat16)
    deq_t, c_t, s_t, z_t = o_pt.quantize_per_token(xt, 8, True)
    out["per_token_int8_sym"] = {"x": xt.float().numpy(), "deq": deq_t.float().numpy(), "codes": c_t.numpy(),
                                 "scales": np.asarray(s_t, np.float32), "zps": np.asarray(z_t, np.int64)}
    # SmoothQuant alpha = 0.5 on bf16 layer norm / q-k-v weights
    am = (torch.rand(256, generator=gen(13)) * 3 + 0.1) * torch.where(torch.rand(256, generator=gen(14)) < 0.03, 25.0, 1.0)
    sw = (1.0 + 0.1 * torch.randn(256, generator=gen(15))).to(torch.bfloat16)
    bw = (torch.randn(384, 256, generator=gen(16)) * 0.02).to(torch.bfloat16)
    ns, nb, sc = o_sq.apply_mapping(sw, bw, am.numpy(), 0.5)
    out["smoothquant_a05"] = {"act_max": am.numpy(), "smooth": sw.float().numpy(), "balance": bw.float().numpy(),
                              "new_smooth": ns.float().numpy(), "new_balance": nb.float().numpy(), "s": sc}
    # AWQ: 20-point grid search, asym int4 g128, on a 64 x 512 bf16 weight
    ww = (torch.randn(64, 512, generator=gen(17)) * 0.02).to(torch.bfloat16)
    aw = (torch.rand(512, generator=gen(18)) * 3 + 0.1) * torch.where(torch.rand(512, generator=gen(19)) < 0.02, 30.0, 1.0)
    rs, rk, rmse = o_awq.awq_search(ww, aw.numpy(), 20, o_rtn.RtnConfig(4, False, "group", group_size=128))
    out["awq_g128"] = {"w": ww.float().numpy(), "act_max": aw.numpy(), "s": np.asarray(rs, np.float32),
                       "k": np.asarray(rk, np.int64), "mse": np.asarray(rmse, np.float64)}
    return out


def main(names=None):
    """Writes every fixture, or only ``names`` (so that the others keep their bytes)."""
    for name, arrays in cases().items():
        if names and name not in names:
            continue
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        print(name, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main(sys.argv[1:])
