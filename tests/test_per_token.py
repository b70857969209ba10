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


@pytest.mark.parametrize("bits,sym", [(8, True), (8, False), (4, True), (4, False)])
@pytest.mark.parametrize("rows,cols", [(333, 4096), (1000, 2048), (64, 256), (50, 768)])
def test_per_token_codes_only_bf16_rows_in_registers(bits, sym, rows, cols):
    """Codes without fake-quantised values for bf16 rows of up to 4,096 columns (a multiple of
    256) take the register-resident kernel; codes, scales and zero-points equal the oracle's.
    A few hundred thousand elements per case put some quotients near a bf16 rounding midpoint,
    the elements that kernel hands to the op-by-op chain; a row of exact midpoints forces it."""
    from llmcompressorsharp_b200 import quantize_per_token

    x = acts(rows, cols, torch.bfloat16, rows + cols + bits)
    if rows > 5:
        # symmetric grids: absmax 63.5 (int8) or 3.5 (int4) gives scale 1/2, so the other
        # entries, (k + 1/2) / 2, divide to exact half-integers (ties of the rounding)
        half = 127.0 if bits == 8 else 7.0
        x[5] = (((torch.arange(cols) % 8) - 4.0) * 0.5 + 0.25).to(torch.bfloat16)
        x[5, 0] = half / 2
    codes, scales, zps, deq = quantize_per_token(x.to(DEV), bits, sym, want_values=False)
    assert deq is None
    rdeq, rcodes, rs, rz = o_pt.quantize_per_token(x, bits, sym)
    assert np.array_equal(scales.cpu().numpy(), rs)
    assert np.array_equal(zps.cpu().numpy(), rz.astype(np.int32))
    assert torch.equal(codes.cpu().to(torch.int32), rcodes)


def test_per_token_codes_only_nan_row_bf16():
    """A NaN row has NaN parameters; its codes have no reference meaning (the fake-quantised
    values are NaN), so they are only checked to be the same bytes the values path writes."""
    from llmcompressorsharp_b200 import quantize_per_token

    x = acts(24, 1024, torch.bfloat16, 77)
    x[3, 100] = float("nan")
    codes, scales, _, _ = quantize_per_token(x.to(DEV), 8, True)
    codes_v, _, _, _ = quantize_per_token(x.to(DEV), 8, True, want_values=True)
    _, rcodes, rs, _ = o_pt.quantize_per_token(x, 8, True)
    assert np.array_equal(scales.cpu().numpy(), rs, equal_nan=True)
    ok = torch.ones(24, dtype=torch.bool)
    ok[3] = False
    assert torch.equal(codes.cpu().to(torch.int32)[ok], rcodes[ok])
    assert torch.equal(codes.cpu()[3], codes_v.cpu()[3])
