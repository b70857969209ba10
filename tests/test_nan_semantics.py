"""NaN in calibration data: the CUDA observers, RTN and GPTQ parameters follow the reference.

  * MinMaxObserver (MinMaxObserver.cs:29-42): x.min() of a batch holding a NaN is NaN and
    `NaN < _min` is false, so the batch changes neither running value (a first such batch
    leaves +inf / -inf).
  * PerChannelMinMaxObserver (PerChannelMinMaxObserver.cs:55-74): amin / amax and
    torch.minimum / maximum propagate NaN per channel.
  * MovingAverageMinMaxObserver (MovingAverageMinMaxObserver.cs:44-60) averages the raw batch
    values, NaN included.
  * GPTQ's ComputeScaleZeroPoint builds a new MinMaxObserver per tensor or row
    (GptqBlockQuantizer.cs:200-230), so a NaN row gets the parameters of (+inf, -inf).
Every check compares with the oracle; NaN positions must match (np.array_equal(equal_nan=True))."""

import numpy as np
import pytest
import torch

from oracle import affine as o_aff, gptq as o_gptq, rtn as o_rtn

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
NAN = float("nan")


def _np(a):
    if torch.is_tensor(a):  # bf16 / f16 widen to fp32 exactly (NaN stays NaN)
        a = a.detach().cpu()
        a = a.float() if a.is_floating_point() else a
        return a.numpy().astype(np.float64)
    return np.asarray(a, dtype=np.float64)


def same(a, b):
    a, b = _np(a), _np(b)
    return a.shape == b.shape and np.array_equal(a, b, equal_nan=True)


def nan_weight(m, n, dtype, seed=3):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(m, n, generator=g) * 0.02
    w[1, 5] = NAN
    w[m - 1, n - 1] = NAN
    return w.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_minmax_observer_nan_batches(dtype):
    from llmcompressorsharp_b200 import MinMaxObserver

    batches = [torch.tensor([[-2.0, NAN, 3.0]]), torch.tensor([[-1.0, 4.0, 0.5]]),
               torch.tensor([[NAN, -9.0, 9.0]]), torch.tensor([[-1.5, 2.0, 0.0]])]
    dev, ref = MinMaxObserver(DEV), o_aff.MinMaxObserver()
    for i, b in enumerate(batches):
        dev.update(b.to(dtype).to(DEV))
        ref.update(b.to(dtype))
        mn, mx = dev.min_max()
        assert same([mn, mx], [ref._min, ref._max]), (i, mn, mx, ref._min, ref._max)
    for bits, sym in ((8, True), (4, False)):
        assert dev.get_quant_params(bits, sym) == pytest.approx(ref.get_quant_params(bits, sym), rel=0, abs=0)


def test_minmax_observer_only_nan_batches_keep_infinities():
    from llmcompressorsharp_b200 import MinMaxObserver

    dev = MinMaxObserver(DEV)
    dev.update(torch.tensor([NAN, 1.0], device=DEV))
    assert dev.min_max() == (float("inf"), float("-inf"))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_per_channel_and_group_observers_propagate_nan(dtype):
    from llmcompressorsharp_b200 import GroupMinMaxObserver, PerChannelMinMaxObserver

    a, b = nan_weight(40, 384, dtype, 1), nan_weight(40, 384, dtype, 2)
    b[1, 5] = 0.0  # channel 1 saw its NaN in the first batch only: it stays NaN
    pc, rpc = PerChannelMinMaxObserver(0), o_aff.PerChannelMinMaxObserver(0)
    for x in (a, b):
        pc.update(x.to(DEV))
        rpc.update(x)
    assert same(pc._min, rpc._min) and same(pc._max, rpc._max)
    assert np.isnan(pc._min[1].item())
    s, z = pc.get_quant_params(4, False)
    rs, rz = rpc.get_quant_params(4, False)
    assert same(s, rs) and same(z, rz)
    go = GroupMinMaxObserver(128)
    go.update(a.to(DEV))
    mins, maxs = o_aff.group_minmax(a, 128)
    assert same(go._min, mins) and same(go._max, maxs)


def test_moving_average_observer_takes_raw_nan_batch():
    from llmcompressorsharp_b200 import MovingAverageMinMaxObserver

    dev, ref = MovingAverageMinMaxObserver(0.5, DEV), o_aff.MovingAverageMinMaxObserver(0.5)
    for b in (torch.tensor([-1.0, 2.0]), torch.tensor([NAN, 3.0])):
        dev.update(b.to(DEV))
        ref.update(b)
    assert same([dev._min, dev._max], [ref._min, ref._max])
    assert np.isnan(dev._min)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("strategy", ["tensor", "channel", "group"])
@pytest.mark.parametrize("shape", [(37, 300), (64, 4096)])
def test_rtn_parameters_and_values_with_nan(dtype, strategy, shape):
    from llmcompressorsharp_b200 import RtnConfig, rtn_quantize

    m, n = shape
    w = nan_weight(m, n, dtype)
    gs = 128 if n % 128 == 0 else 100
    for bits, sym in ((4, False), (8, True)):
        deq, _, scales, zps = rtn_quantize(w.to(DEV), RtnConfig(num_bits=bits, symmetric=sym, strategy=strategy,
                                                                 group_size=gs))
        rdeq, _, rs, rz = o_rtn.rtn_quantize(w, o_rtn.RtnConfig(bits, sym, strategy, group_size=gs))
        k = 1 if strategy == "tensor" else None
        assert same(scales.reshape(-1), np.asarray(rs, np.float32).reshape(-1)[:k])
        assert same(zps.reshape(-1), np.asarray(rz).reshape(-1)[:k])
        assert same(deq, rdeq)


@pytest.mark.parametrize("strategy", ["tensor", "channel", "group"])
def test_gptq_parameters_of_nan_rows(strategy):
    from llmcompressorsharp_b200 import GPTQConfig, gptq_quantize_u

    m, n = 64, 256
    w = nan_weight(m, n, torch.float32)
    u = torch.eye(n)
    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy=strategy, group_size=128, block_size=128)
    res = gptq_quantize_u(w.to(DEV), u.to(DEV), cfg)
    rs, rz = o_gptq.compute_scale_zero_point(
        w, o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy=strategy, group_size=128, block_size=128))
    k = 1 if strategy == "tensor" else None
    got_s = res.scales.reshape(-1).cpu().numpy()
    got_z = res.zero_points.reshape(-1).cpu().numpy()
    assert same(got_s[:k] if k else got_s, np.asarray(rs, np.float32).reshape(-1)[:k] if k else rs.reshape(-1))
    assert same(got_z[:k] if k else got_z, np.asarray(rz).reshape(-1)[:k] if k else rz.reshape(-1))
