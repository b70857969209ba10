"""Pins the CPU oracle to the known-answer values in the reference's own xUnit tests.

Each test cites the reference test it ports (tests/LLMCompressorSharp.Tests/...).  The
oracle is the checker for every GPU parity test, so these run first and on the CPU.
"""

import numpy as np
import pytest
import torch

from oracle import affine, fakequant, gptq, hessian, rtn, smoothquant

T = "tests/LLMCompressorSharp.Tests/"


# --- HessianAccumulatorTests.cs -------------------------------------------------------

def test_hessian_initial_zero():  # HessianAccumulatorTests.cs:16-25
    acc = hessian.HessianAccumulator(4)
    assert acc.sample_count == 0
    h = acc.get_hessian()
    assert h.shape == (4, 4) and torch.count_nonzero(h) == 0


def test_hessian_one_batch_outer_product():  # :27-43
    acc = hessian.HessianAccumulator(3)
    acc.update(torch.tensor([[1.0, 2.0, 3.0]]))
    assert acc.sample_count == 1
    assert acc.get_hessian().flatten().tolist() == [1, 2, 3, 2, 4, 6, 3, 6, 9]


def test_hessian_multiple_batches_additive():  # :45-58
    acc = hessian.HessianAccumulator(2)
    acc.update(torch.tensor([[1.0, 0.0]]))
    acc.update(torch.tensor([[0.0, 1.0]]))
    assert acc.sample_count == 2
    assert acc.get_hessian().flatten().tolist() == [1, 0, 0, 1]


def test_hessian_high_rank_flattens():  # :60-83
    acc = hessian.HessianAccumulator(2)
    blk = [[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]]
    acc.update(torch.tensor([blk, blk]))
    assert acc.sample_count == 6
    assert acc.get_hessian().flatten().tolist() == [4, 2, 2, 4]


def test_hessian_wrong_in_features_throws():  # :85-92
    acc = hessian.HessianAccumulator(3)
    with pytest.raises(ValueError, match="last dim"):
        acc.update(torch.tensor([[1.0, 2.0]]))


def test_hessian_fp16_input_accumulates_fp32():  # :94-103
    acc = hessian.HessianAccumulator(2)
    acc.update(torch.tensor([[1.0, 2.0]]).to(torch.float16))
    assert acc.get_hessian().dtype == torch.float32


def test_hessian_reset():  # :105-116
    acc = hessian.HessianAccumulator(2)
    acc.update(torch.tensor([[1.0, 2.0]]))
    acc.reset()
    assert acc.sample_count == 0 and torch.count_nonzero(acc.get_hessian()) == 0


def test_hessian_nonpositive_in_features_throws():  # :118-123
    with pytest.raises(ValueError):
        hessian.HessianAccumulator(0)


# --- HessianInverseSolverTests.cs ----------------------------------------------------

def test_inverse_identity():  # HessianInverseSolverTests.cs:17-27
    hinv = hessian.hessian_inverse(torch.eye(4), 0.0)
    assert (hinv - torch.eye(4)).abs().max() < 1e-5


def test_inverse_scaled_identity():  # :29-39
    hinv = hessian.hessian_inverse(2 * torch.eye(3), 0.0)
    assert (hinv - 0.5 * torch.eye(3)).abs().max() < 1e-5


def test_inverse_rank_deficient_damped_finite():  # :41-51
    assert torch.isfinite(hessian.hessian_inverse(torch.ones(2, 2), 0.01)).all()


def test_inverse_ill_conditioned_finite():  # :53-63
    assert torch.isfinite(hessian.hessian_inverse(torch.eye(4) * 1e-10, 0.0)).all()


def test_inverse_non_square_throws():  # :72-78
    with pytest.raises(ValueError, match="square"):
        hessian.hessian_inverse(torch.ones(3, 4), 0.01)


def test_inverse_output_fp32_and_no_alias():  # :80-101
    h = torch.eye(3)
    hinv = hessian.hessian_inverse(h, 0.01)
    assert hinv.dtype == torch.float32
    h.fill_(float("nan"))
    assert torch.isfinite(hinv).all()


# --- MinMaxObserverTests.cs ----------------------------------------------------------

def test_minmax_accumulates_asym():  # MinMaxObserverTests.cs:22-42
    obs = affine.MinMaxObserver()
    for b in ([-2.0, 0.0, 3.0], [-5.0, 1.0, 2.0], [-1.0, 7.0, 0.0]):
        obs.update(torch.tensor(b))
    s, z = obs.get_quant_params(8, False)
    assert abs(s - 12 / 255) < 1e-5
    assert z == 106


def test_minmax_symmetric():  # :44-58
    obs = affine.MinMaxObserver()
    obs.update(torch.tensor([-3.0, 0.0, 5.0]))
    s, z = obs.get_quant_params(8, True)
    assert abs(s - 5 / 127) < 1e-5 and z == 0


def test_minmax_reset():  # :60-74
    obs = affine.MinMaxObserver()
    obs.update(torch.tensor([-10.0, 10.0]))
    obs.reset()
    obs.update(torch.tensor([-1.0, 1.0]))
    assert abs(obs.get_quant_params(8, True)[0] - 1 / 127) < 1e-5


def test_minmax_no_samples_throws():  # :76-83
    with pytest.raises(RuntimeError, match="no calibration samples"):
        affine.MinMaxObserver().get_quant_params(8, True)


def test_minmax_all_zeros_scale_one():  # :85-95
    obs = affine.MinMaxObserver()
    obs.update(torch.zeros(3))
    assert obs.get_quant_params(8, True) == (1.0, 0)


# Derived from the code (no reference test): a batch holding a NaN has x.min() = x.max() = NaN,
# `NaN < _min` is false, so MinMaxObserver.Update (MinMaxObserver.cs:29-42) leaves both running
# values as they were; a first NaN batch leaves +inf / -inf.
def test_minmax_nan_batch_changes_nothing():
    obs = affine.MinMaxObserver()
    obs.update(torch.tensor([-2.0, float("nan"), 3.0]))
    assert obs._min == np.float32(np.inf) and obs._max == np.float32(-np.inf)
    obs.update(torch.tensor([-1.0, 4.0]))
    obs.update(torch.tensor([float("nan"), -9.0, 9.0]))
    assert (obs._min, obs._max) == (np.float32(-1.0), np.float32(4.0))
    assert obs.get_quant_params(8, True) == pytest.approx((4 / 127, 0))


# MathF.Max(MathF.Abs(NaN), x) is NaN, so ComputeAffineParams (Observer.cs:58-75) gives a NaN
# scale; NaN zero-points saturate to 0.
def test_affine_params_nan_inputs():
    s, z = affine.compute_affine_params(float("nan"), 1.0, 8, True)
    assert np.isnan(s) and z == 0
    s, z = affine.compute_affine_params(1.0, float("nan"), 8, True)
    assert np.isnan(s) and z == 0
    s, z = affine.compute_affine_params(float("nan"), 1.0, 4, False)
    assert np.isnan(s) and z == 0


# --- PerChannelMinMaxObserverTests.cs ------------------------------------------------

# Derived: amin / amax and torch.minimum / maximum propagate NaN
# (PerChannelMinMaxObserver.cs:55-74), so a channel that ever saw a NaN stays NaN.
def test_per_channel_nan_propagates():
    obs = affine.PerChannelMinMaxObserver(0)
    obs.update(torch.tensor([[-1.0, float("nan")], [-3.0, 5.0]]))
    obs.update(torch.tensor([[-5.0, 1.0], [-2.0, 8.0]]))
    assert np.isnan(obs._min[0].item()) and np.isnan(obs._max[0].item())
    assert obs._min[1].item() == -3.0 and obs._max[1].item() == 8.0


# Derived: ComputeScaleZeroPoint builds a new MinMaxObserver per row (GptqBlockQuantizer.cs:212-222),
# so a weight row holding a NaN is quantised with the parameters of (+inf, -inf).
def test_gptq_params_of_a_nan_row_follow_the_observer():
    w = torch.tensor([[1.0, float("nan"), -2.0, 0.5], [0.25, -0.5, 1.0, -1.0]])
    s, z = gptq.compute_scale_zero_point(w, gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="channel"))
    ref = affine.compute_affine_params(np.inf, -np.inf, 4, False)
    assert (np.isnan(s[0, 0]) and np.isnan(ref[0])) or s[0, 0] == ref[0]
    assert z[0, 0] == ref[1]
    assert (s[1, 0], z[1, 0]) == affine.compute_affine_params(-1.0, 1.0, 4, False)


def test_per_channel_one_scale_per_row():  # PerChannelMinMaxObserverTests.cs:118-143
    obs = affine.PerChannelMinMaxObserver(0)
    obs.update(torch.tensor([[-2.0, 0.0, 4.0], [-10.0, 5.0, 10.0]]))
    s, z = obs.get_quant_params(8, True)
    assert s.shape == (2,)
    assert abs(s[0] - 4 / 127) < 1e-5 and abs(s[1] - 10 / 127) < 1e-5


def test_per_channel_accumulates():  # :145-171
    obs = affine.PerChannelMinMaxObserver(0)
    obs.update(torch.tensor([[-1.0, 2.0], [-3.0, 5.0]]))
    obs.update(torch.tensor([[-5.0, 1.0], [-2.0, 8.0]]))
    s, _ = obs.get_quant_params(8, True)
    assert abs(s[0] - 5 / 127) < 1e-5 and abs(s[1] - 8 / 127) < 1e-5


def test_per_channel_reset_and_errors():  # :173-219
    obs = affine.PerChannelMinMaxObserver(0)
    with pytest.raises(RuntimeError):
        obs.get_quant_params(8, True)
    obs.update(torch.tensor([[-10.0, 10.0], [-20.0, 20.0]]))
    obs.reset()
    obs.update(torch.tensor([[-1.0, 1.0], [-2.0, 2.0]]))
    s, _ = obs.get_quant_params(8, True)
    assert abs(s[0] - 1 / 127) < 1e-5 and abs(s[1] - 2 / 127) < 1e-5
    with pytest.raises(IndexError):
        affine.PerChannelMinMaxObserver(5).update(torch.ones(2, 2))


# --- MovingAverageMinMaxObserverTests.cs / MSEObserverTests.cs ------------------------

def test_ema_observer():  # MovingAverageMinMaxObserverTests.cs:23-50
    obs = affine.MovingAverageMinMaxObserver(0.5)
    obs.update(torch.tensor([-3.0, 7.0]))
    assert abs(obs.get_quant_params(8, True)[0] - 7 / 127) < 1e-5
    obs = affine.MovingAverageMinMaxObserver(0.5)
    obs.update(torch.tensor([-10.0, 10.0]))
    obs.update(torch.tensor([-2.0, 2.0]))
    assert abs(obs.get_quant_params(8, True)[0] - 6 / 127) < 1e-5
    with pytest.raises(ValueError):
        affine.MovingAverageMinMaxObserver(1.5)


def test_mse_observer():  # MSEObserverTests.cs:38-66
    obs = affine.MSEObserver(80)
    obs.update(torch.tensor([-3.0, -2.5, -1.0, 0.0, 1.0, 2.5, 3.0]))
    s, _ = obs.get_quant_params(8, True)
    assert 0.001 <= s <= 0.5
    vals = [i / 98 for i in range(99)] + [1.5]
    mse, mm = affine.MSEObserver(100), affine.MinMaxObserver()
    mse.update(torch.tensor(vals))
    mm.update(torch.tensor(vals))
    assert mse.get_quant_params(4, True)[0] < mm.get_quant_params(4, True)[0]


def test_affine_bits_out_of_range():  # Observer.cs:53-56
    with pytest.raises(ValueError):
        affine.compute_affine_params(-1, 1, 1, True)


# --- FakeQuantizeFunctionTests.cs ----------------------------------------------------

def test_fake_quant_sym8():  # FakeQuantizeFunctionTests.cs:16-30
    y = fakequant.fake_quantize(torch.tensor([-127.4, -127.6, 0.4, 0.6, 127.4, 127.6]), 1.0, 0, 8, True)
    assert y.tolist() == [-127, -127, 0, 1, 127, 127]


def test_fake_quant_sym4_scale():  # :32-43
    y = fakequant.fake_quantize(torch.tensor([-3.6, 0.0, 3.6]), 0.5, 0, 4, True)
    assert y.tolist() == [-3.5, 0.0, 3.5]


def test_fake_quant_asym_zero_point():  # :60-73
    y = fakequant.fake_quantize(torch.tensor([-8.0, 0.0, 7.0]), 1.0, 8, 4, False)
    assert y.tolist() == [-8.0, 0.0, 7.0]


def test_fake_quant_invalid_bits():  # :75-81
    with pytest.raises(ValueError):
        fakequant.fake_quantize(torch.tensor([1.0, 2.0]), 1.0, 0, 1, True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fake_quant_restates_libtorch_chain(dtype):
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(200_000, generator=g) * 0.05).to(dtype)
    for bits, sym in ((4, True), (4, False), (8, True), (8, False)):
        s = np.float32(0.0071234)
        z = 0 if sym else 7
        a = fakequant.fake_quantize(x, float(s), z, bits, sym)
        b = fakequant.fake_quantize_torch_chain(x, float(s), z, bits, sym)
        assert a.dtype == b.dtype == dtype
        assert torch.equal(a, b)


# --- Int4PackedTensorTests.cs --------------------------------------------------------

def test_int4_clamps_symmetric():  # Int4PackedTensorTests.cs:16-31
    p = fakequant.Int4PackedTensor.from_float(torch.tensor([-8.5, -7.0, 0.0, 7.0, 9.0]), 1.0, 0, True)
    assert p.dequantize().tolist() == [-7, -7, 0, 7, 7]


def test_int4_halves_storage():  # :33-41
    p = fakequant.Int4PackedTensor.from_float(torch.arange(1.0, 9.0), 1.0, 0, True)
    assert len(p.packed_bytes) == 4


def test_int4_round_trip():  # :43-59
    vals = [-7.0, -3.0, 0.0, 4.0, 7.0, -2.0]
    p = fakequant.Int4PackedTensor.from_float(torch.tensor(vals), 1.0, 0, True)
    r = fakequant.Int4PackedTensor.from_packed_bytes(p.packed_bytes, 6, 1.0, 0, True)
    assert r.dequantize().tolist() == vals


def test_int4_asymmetric():  # :61-68
    p = fakequant.Int4PackedTensor.from_float(torch.tensor([-8.0, 0.0, 7.0]), 1.0, 8, False)
    assert p.dequantize().tolist() == [-8, 0, 7]


def test_int4_nibble_order():  # Int4PackedTensor.cs:52-64 — even index in the high nibble
    p = fakequant.Int4PackedTensor.from_float(torch.tensor([1.0, 2.0, -1.0]), 1.0, 0, True)
    assert p.packed_bytes == bytes([0x12, 0xF0])
    rows = fakequant.pack_int4_rows(torch.tensor([[1, 2, -1]]))
    assert rows.flatten().tolist() == [0x12, 0xF0]


# --- RtnModifierTests.cs -------------------------------------------------------------

def test_rtn_sym8_grid():  # RtnModifierTests.cs:22-49
    w = torch.tensor([-127.0, -64.4, 0.0, 64.6, 127.0, 127.0])
    out, codes, _, _ = rtn.rtn_quantize(w, rtn.RtnConfig(8, True, "tensor"))
    assert out.tolist() == [-127, -64, 0, 65, 127, 127]


def test_rtn_per_channel():  # :51-79
    w = torch.tensor([[-2.0, 0.0, 2.0], [-10.0, 5.0, 10.0]])
    out, _, _, _ = rtn.rtn_quantize(w, rtn.RtnConfig(8, True, "channel"))
    assert abs(out[0, 0] + 2) < 1e-4 and abs(out[0, 2] - 2) < 1e-4
    assert abs(out[1, 0] + 10) < 1e-4 and abs(out[1, 2] - 10) < 1e-4


def test_rtn_int4_targets_value():  # :81-109 (the quantised weight's values)
    out, _, _, _ = rtn.rtn_quantize(torch.tensor([-10.0, 0.0, 10.0]), rtn.RtnConfig(4, True, "tensor"))
    assert abs(out[0] + 10) <= 2 and abs(out[1]) <= 2


def test_rtn_asym8():  # :111-133
    out, _, _, _ = rtn.rtn_quantize(torch.tensor([-1.0, 0.0, 3.0, 7.0]), rtn.RtnConfig(8, False, "tensor"))
    assert abs(out[0] + 1) < 0.1 and abs(out[1]) < 0.1 and abs(out[3] - 7) < 0.1


def test_rtn_per_token_rejected():  # RtnModifier.cs:69-70
    with pytest.raises(NotImplementedError):
        rtn.rtn_quantize(torch.ones(2, 2), rtn.RtnConfig(8, True, "token"))


# --- GptqBlockQuantizerTests.cs / GPTQModifierTests.cs --------------------------------

def _cfg(bits=8, bs=128, strategy="tensor"):
    return gptq.GPTQConfig(num_bits=bits, symmetric=True, strategy=strategy, block_size=bs)


def test_gptq_zero_weight():  # GptqBlockQuantizerTests.cs:18-30
    wq, *_ = gptq.gptq_quantize(torch.zeros(2, 4), torch.eye(4), _cfg(8))
    assert wq.abs().max() < 1e-6


def test_gptq_shapes_and_finite():  # :32-83
    g = torch.Generator().manual_seed(1)
    for (m, n, bits, bs) in ((4, 8, 4, 128), (3, 6, 4, 2), (2, 6, 8, 128)):
        w = torch.randn(m, n, generator=g)
        wq, *_ = gptq.gptq_quantize(w, torch.eye(n), _cfg(bits, bs))
        assert wq.shape == w.shape and torch.isfinite(wq).all()


def test_gptq_16bit_identity():  # :57-69 and :115-138
    g = torch.Generator().manual_seed(2)
    w = torch.randn(2, 4, generator=g)
    wq, *_ = gptq.gptq_quantize(w, torch.eye(4), _cfg(16, 4))
    assert (w - wq).abs().max() < 1e-3
    w = torch.tensor([[1.0, 2.0], [3.0, 4.0]])
    wq, *_ = gptq.gptq_quantize(w, torch.eye(2), _cfg(16, 1))
    assert torch.allclose(wq, w, atol=0.01)


def test_gptq_act_order_throws():  # GPTQModifierTests.cs:130-141
    with pytest.raises(NotImplementedError, match="ActOrder"):
        gptq.gptq_quantize(torch.ones(2, 2), torch.eye(2), gptq.GPTQConfig(act_order=True))


def test_gptq_no_batches_is_rtn():  # GPTQModifierTests.cs:92-110: H = 0 -> pinv -> U = Hinv -> zero pivots
    g = torch.Generator().manual_seed(3)
    w = torch.randn(3, 4, generator=g)
    hinv = hessian.hessian_inverse(torch.zeros(4, 4), 0.01)
    assert torch.count_nonzero(hinv) == 0
    cfg = gptq.GPTQConfig(num_bits=8, symmetric=True, strategy="tensor", block_size=4)
    wq, *_ = gptq.gptq_quantize(w, hinv, cfg)
    out, *_ = rtn.rtn_quantize(w, rtn.RtnConfig(8, True, "tensor"))
    assert torch.equal(wq, out)


def test_inverse_singular_is_pinv():  # derived KAT, HessianInverseSolver.cs:85-91: no Cholesky factor -> pinv(H')
    h = torch.diag(torch.tensor([2.0, 0.0, 4.0, 0.0]))
    assert torch.allclose(hessian.hessian_inverse(h, 0.0), torch.diag(torch.tensor([0.5, 0.0, 0.25, 0.0])), atol=1e-7)
    neg = -torch.eye(3)  # indefinite: pinv is the inverse, and U falls back to Hinv (GptqBlockQuantizer.cs:112-118)
    hinv = hessian.hessian_inverse(neg, 0.0)
    assert torch.allclose(hinv, -torch.eye(3), atol=1e-7)
    assert torch.equal(hessian.upper_factor(hinv), hinv)


def test_gptq_identity_hinv_is_rtn():  # derived KAT: Hinv = I -> U = I -> no cross-column coupling
    g = torch.Generator().manual_seed(4)
    w = torch.randn(16, 40, generator=g)
    for strategy in ("tensor", "channel", "group"):
        cfg = gptq.GPTQConfig(num_bits=4, symmetric=False, strategy=strategy, block_size=16, group_size=8)
        wq, codes, _, _ = gptq.gptq_quantize(w, torch.eye(40), cfg)
        out, rcodes, _, _ = rtn.rtn_quantize(w, rtn.RtnConfig(4, False, strategy, group_size=8))
        assert torch.equal(wq, out) and torch.equal(codes, rcodes)


def test_gptq_reduces_reconstruction_error():  # GPTQ's purpose: lower ||dW X|| than RTN
    g = torch.Generator().manual_seed(5)
    x = torch.randn(512, 64, generator=g) @ torch.randn(64, 64, generator=g) * 0.3
    acc = hessian.HessianAccumulator(64)
    acc.update(x)
    h = acc.get_hessian()
    w = torch.randn(32, 64, generator=g) * 0.02
    cfg = gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=32, block_size=32)
    wq, *_ = gptq.gptq_quantize(w, hessian.hessian_inverse(h, 0.01), cfg)
    rq, *_ = rtn.rtn_quantize(w, rtn.RtnConfig(4, False, "group", group_size=32))
    assert gptq.reconstruction_error(w, wq, h) < 0.8 * gptq.reconstruction_error(w, rq, h)


# --- SmoothQuantModifierTests.cs -----------------------------------------------------

def test_smoothquant_exact_weights():  # SmoothQuantModifierTests.cs:26-73
    amax = smoothquant.update_running_max(None, torch.tensor([[1.0, 4.0], [-0.5, -2.0]]))
    g, w, _ = smoothquant.apply_mapping(torch.tensor([2.0, 4.0]), torch.ones(2, 2), amax, 0.5)
    assert torch.allclose(g, torch.tensor([2.0, 2.0]), atol=1e-4)
    assert torch.allclose(w, torch.tensor([[1.0, 2.0], [1.0, 2.0]]), atol=1e-4)


def test_smoothquant_identity_preserved():  # :75-123
    g = torch.tensor([1.0, 2.0, 3.0])
    w = torch.tensor([[0.5, 1.0, -1.0], [2.0, -0.5, 0.25]])
    x = torch.tensor([[0.1, 0.5, -1.0], [0.2, -0.3, 0.7]])
    y_ref = (x * g) @ w.t()
    amax = smoothquant.update_running_max(None, x * g)
    g2, w2, _ = smoothquant.apply_mapping(g, w, amax, 0.5)
    assert torch.allclose((x * g2) @ w2.t(), y_ref, atol=1e-4)


def test_smoothquant_errors():  # :125-152, ApplyMapping checks :142-158
    with pytest.raises(RuntimeError, match="1-D"):
        smoothquant.apply_mapping(torch.ones(1, 2), torch.ones(1, 2), np.ones(2, np.float32), 0.5)
    with pytest.raises(RuntimeError, match="changed"):
        smoothquant.update_running_max(np.ones(2, np.float32), torch.ones(2, 3))
