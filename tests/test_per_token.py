"""Dynamic per-token activation quantisation (extension, parity unpinned) against the oracle's
restatement (oracle/pertoken.py): scales, zero-points, codes and fake-quantised values bit-exact
for every dtype, symmetric and asymmetric grids, aligned (16-byte vector) and unaligned shapes,
rows with outliers and a row holding a NaN."""

import numpy as np
import pytest
import torch

from oracle import pertoken as o_pt

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def acts(rows, cols, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * torch.exp(torch.randn(rows, 1, generator=g))
    x[0, 3] = 60.0  # outlier row
    if rows > 2:
        x[2] = 0.0  # all-zero row: scale 1
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("bits,sym", [(8, True), (8, False), (4, True), (6, False)])
@pytest.mark.parametrize("rows,cols", [(333, 4096), (64, 1000), (7, 37)])
def test_per_token_bit_exact(dtype, bits, sym, rows, cols):
    from llmcompressorsharp_b200 import quantize_per_token

    x = acts(rows, cols, dtype, rows * cols + bits)
    codes, scales, zps, deq = quantize_per_token(x.to(DEV), bits, sym, want_values=True)
    rdeq, rcodes, rs, rz = o_pt.quantize_per_token(x, bits, sym)
    assert np.array_equal(scales.cpu().numpy(), rs)
    assert np.array_equal(zps.cpu().numpy(), rz.astype(np.int32))
    assert torch.equal(deq.cpu(), rdeq)
    got = codes.cpu().to(torch.int32)
    assert torch.equal(got, rcodes)


def test_per_token_nan_row_and_strided_input():
    from llmcompressorsharp_b200 import quantize_per_token

    base = torch.randn(40, 520, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    x = base[:, 4:516]
    x[5, 7] = float("nan")
    xd = base.to(DEV)[:, 4:516]  # the same view on the device: row stride 520, start 8 bytes in
    codes, scales, zps, deq = quantize_per_token(xd, 8, True, want_values=True)
    rdeq, rcodes, rs, rz = o_pt.quantize_per_token(x.contiguous(), 8, True)
    assert np.array_equal(scales.cpu().numpy(), rs, equal_nan=True)
    assert np.isnan(scales[5].item())
    ok = torch.ones(40, dtype=torch.bool)
    ok[5] = False
    assert torch.equal(deq.cpu()[ok], rdeq[ok])
    assert torch.isnan(deq.cpu()[5]).all()
    assert torch.equal(codes.cpu().to(torch.int32)[ok], rcodes[ok])


def test_per_token_rejects_wide_codes():
    from llmcompressorsharp_b200 import ArgumentOutOfRangeError, quantize_per_token

    with pytest.raises(ArgumentOutOfRangeError):
        quantize_per_token(torch.ones(2, 8, device=DEV), 9, True)
