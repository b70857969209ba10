"""Bounded device waits of the tensor-core kernels: a wait that runs out stops the kernel,
the context reports LLMC_ERR_TIMEOUT once, and the next call on the same context works.

The limit is set to 0 tries (llmc_set_wait_limit), so the first wait of each kernel gives up
before the kernel has issued any copy or MMA: no GPU fault or hang is involved, only the
abort path's error word, its tensor-memory release and the host's status reporting.  Each
case runs on a context of its own, bound to torch's current stream."""

import ctypes as C

import pytest
import torch

from llmcompressorsharp_b200 import _lib
from oracle import hessian as o_hess

pytestmark = pytest.mark.gpu

TIMEOUT = 7  # LLMC_ERR_TIMEOUT


def _ctx():
    lib = _lib.load()
    c = C.c_void_p()
    assert lib.llmc_init(0, C.byref(c)) == 0, _lib.last_error()
    assert lib.llmc_set_stream(c, C.c_void_p(torch.cuda.current_stream().cuda_stream or 1)) == 0
    return lib, c


def _hessian(lib, c, x):
    d = x.shape[1]
    h = C.c_void_p()
    assert lib.llmc_hessian_create(c, d, C.byref(h)) == 0, _lib.last_error()
    return h


def _update(lib, h, x):
    return lib.llmc_hessian_update(h, C.c_void_p(x.data_ptr()), _lib.dtype_code(x.dtype), x.shape[0], x.stride(0))


def _get(lib, h, d):
    out = torch.empty(d, d, device="cuda")
    st = lib.llmc_hessian_get(h, C.c_void_p(out.data_ptr()))
    return st, out


@pytest.mark.parametrize("d,rows,dtype", [
    (128, 1024, torch.bfloat16),   # one-CTA tcgen05 kernel
    (512, 4096, torch.bfloat16),   # CTA-pair kernel, dynamic unit order
    (512, 2048, torch.float32),    # 3xTF32 pair GEMM
])
def test_wait_limit_zero_times_out_and_context_recovers(d, rows, dtype):
    lib, c = _ctx()
    try:
        x = torch.randn(rows, d, generator=torch.Generator().manual_seed(d + rows)).to(dtype)
        xd = x.cuda()
        h = _hessian(lib, c, xd)
        assert lib.llmc_set_wait_limit(c, 0) == 0
        assert _update(lib, h, xd) == 0, _lib.last_error()  # enqueued; the kernel gives up
        assert lib.llmc_sync(c) == TIMEOUT
        assert "bounded wait" in _lib.last_error()
        assert lib.llmc_sync(c) == 0  # the error word was cleared
        # Default limit again: the same context and handle give the oracle's Hessian.
        assert lib.llmc_set_wait_limit(c, -1) == 0
        assert lib.llmc_hessian_reset(h) == 0
        assert _update(lib, h, xd) == 0, _lib.last_error()
        st, got = _get(lib, h, d)
        assert st == 0, _lib.last_error()
        torch.cuda.synchronize()
        ref = o_hess.HessianAccumulator(d)
        ref.update(x)
        want = ref.get_hessian().double()
        err = float((got.cpu().double() - want).norm() / want.norm())
        assert err < 1e-5, err
        assert lib.llmc_hessian_destroy(h) == 0
    finally:
        lib.llmc_destroy(c)


def test_wait_limit_rejects_values_above_32_bits():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib, c = _ctx()
    try:
        assert lib.llmc_set_wait_limit(c, 1 << 33) == 10  # LLMC_ERR_OUT_OF_RANGE
        assert lib.llmc_set_wait_limit(c, 1000) == 0
    finally:
        lib.llmc_destroy(c)
