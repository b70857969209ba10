"""SparseGPT and AWQ as recipe modifiers (extensions registered beside GPTQ / RTN /
SmoothQuant; the reference's registry is AlgorithmsRegistration.cs:22-59): the full lifecycle
(Initialize, OnStart with hooks, OnBatch, OnEnd, Finalize, CompressionSession.cs:44-99) on the
device, against the oracle given the same calibration inputs.  Parity unpinned (the reference
has design documents for both, no code)."""

import numpy as np
import pytest
import torch

from oracle import awq as o_awq, hessian as o_hess, rtn as o_rtn, smoothquant as o_sq, sparsegpt as o_sp

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel_fro(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("structure,sparsity", [("2:4", 0.5), ("unstructured", 0.6)])
def test_sparsegpt_modifier_lifecycle(structure, sparsity):
    from llmcompressorsharp_b200 import CompressionState, SparseGPTConfig, SparseGPTModifier

    torch.manual_seed(3)
    layer = torch.nn.Linear(256, 64, bias=False).to(DEV)
    orig = layer.weight.detach().clone()
    st = CompressionState({"fc.weight": orig.clone(), "other.weight": torch.ones(4, device=DEV)})
    st.named_modules = {"fc": layer}
    cfg = SparseGPTConfig(sparsity=sparsity, mask_structure=structure, block_size=128)
    mod = SparseGPTModifier(cfg)
    mod.initialize(st)
    mod.on_start(st)
    g = torch.Generator(DEV).manual_seed(4)
    xs = [torch.randn(32, 256, device=DEV, generator=g) for _ in range(8)]
    for x in xs:
        layer(x)
        mod.on_batch(st)
    mod.on_end(st)
    mod.finalize(st)
    assert torch.equal(st.named_weights["other.weight"], torch.ones(4, device=DEV))  # no module: skipped
    got = st.named_weights["fc.weight"]
    mask = st.compressed["fc.weight"]["mask"]
    acc = o_hess.HessianAccumulator(256)
    for x in xs:
        acc.update(x.cpu())
    u = o_hess.upper_factor(o_hess.hessian_inverse(acc.get_hessian(), 0.01))
    n_, m_ = cfg.nm()
    rout, rmask = o_sp.sparsegpt_prune_u(orig.cpu(), u, 128, sparsity, n_, m_)
    assert (mask.cpu().bool() == rmask).float().mean() >= 0.999
    assert rel_fro(got, rout) < 1e-3
    assert torch.count_nonzero(got.cpu()[mask.cpu() == 0]) == 0
    if m_:
        assert (mask.cpu().reshape(64, -1, m_).sum(-1) == n_).all()


def test_sparsegpt_modifier_without_batches_leaves_weight():
    from llmcompressorsharp_b200 import CompressionSession, CompressionState, SessionStatus, SparseGPTConfig, SparseGPTModifier

    layer = torch.nn.Linear(64, 16, bias=False).to(DEV)
    w = layer.weight.detach().clone()
    st = CompressionState({"fc.weight": w.clone()})
    st.named_modules = {"fc": layer}
    s = CompressionSession([SparseGPTModifier(SparseGPTConfig())])
    assert s.run(st, []) == SessionStatus.COMPLETED
    assert torch.equal(st.named_weights["fc.weight"], w)


def test_awq_modifier_lifecycle():
    """Two mappings (a LayerNorm-like smooth weight balancing one Linear; a Linear balanced with
    no smooth weight): the modifier's chosen grid point, scale and rewritten weights equal the
    oracle's search on the same running activation maxima."""
    from llmcompressorsharp_b200 import AWQConfig, AWQModifier, CompressionState
    from llmcompressorsharp_b200.smoothquant import SmoothQuantMapping

    g = torch.Generator().manual_seed(12)
    h = 256
    ln = (1.0 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)
    w1 = (torch.randn(128, h, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(64, h, generator=g) * 0.02).to(torch.bfloat16)
    st = CompressionState({"ln.weight": ln.to(DEV), "q.weight": w1.to(DEV), "o.weight": w2.to(DEV)})
    batches = []
    for i in range(3):
        a = torch.randn(16, h, generator=g) * torch.where(torch.rand(h, generator=g) < 0.03, 20.0, 1.0)
        batches.append({"attn_in": a.to(torch.bfloat16), "o_in": (0.5 * a).to(torch.bfloat16)})
    cfg = AWQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, n_grid=20,
                    mappings=[SmoothQuantMapping("ln.weight", "q.weight", "attn_in"),
                              SmoothQuantMapping("", "o.weight", "o_in")])
    mod = AWQModifier(cfg)
    # The caller's calibration loop exposes each batch's activations as state.layer_activations,
    # as for SmoothQuantModifier.OnBatch (SmoothQuantModifier.cs:71-115).
    mod.initialize(st)
    mod.on_start(st)
    for b in batches:
        st.layer_activations = {k: v.to(DEV) for k, v in b.items()}
        mod.on_batch(st)
    mod.on_end(st)
    mod.finalize(st)
    qcfg = o_rtn.RtnConfig(4, False, "group", group_size=128)
    for key, bname, sname, w in (("attn_in", "q.weight", "ln.weight", w1), ("o_in", "o.weight", None, w2)):
        amax = None
        for b in batches:
            amax = o_sq.update_running_max(amax, b[key])
        rs, rk, rmse = o_awq.awq_search(w, amax, 20, qcfg)
        k = mod.chosen[bname]
        assert k == rk or abs(rmse[k - 1] / rmse[rk - 1] - 1) < 1e-4
        if k == rk:
            want_b = (w.to(torch.float32) * rs.unsqueeze(0)).to(torch.bfloat16)
            assert rel_fro(st.named_weights[bname].float(), want_b.float()) < 1e-2
            if sname:
                want_s = (ln.to(torch.float32) / rs).to(torch.bfloat16)
                assert rel_fro(st.named_weights[sname].float(), want_s.float()) < 1e-2
