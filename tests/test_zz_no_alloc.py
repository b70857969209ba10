"""llmc_observer_minmax_tensor_noalloc (per-tensor min/max with a static row buffer) against
the workspace-backed llmc_observer_minmax, both called through the C ABI.

Collected last on purpose (file name), so it also runs after every other GPU test has used
the library; it passes alone as well.  Min/max are exact selections, so the tolerance is
zero."""

import ctypes as C

import pytest
import torch

from llmcompressorsharp_b200 import _lib
from llmcompressorsharp_b200.errors import LlmcError

MAX_ROWS = 65536


def _workspace_path(x, accumulate, mn0=None, mx0=None):
    mn = torch.zeros(1, device=x.device) if mn0 is None else mn0.clone()
    mx = torch.zeros(1, device=x.device) if mx0 is None else mx0.clone()
    _lib.call("llmc_observer_minmax", C.c_void_p(_lib.ctx_for(x.device.index)), _lib.ptr(x), _lib.dtype_code(x.dtype),
              C.c_int64(x.shape[0]), C.c_int64(x.shape[1]), C.c_int64(x.stride(0)), _lib.STRATEGY["tensor"],
              C.c_int64(x.shape[1]), _lib.ptr(mn), _lib.ptr(mx), accumulate)
    return mn, mx


def _noalloc_path(x, accumulate, mn0=None, mx0=None):
    mn = torch.zeros(1, device=x.device) if mn0 is None else mn0.clone()
    mx = torch.zeros(1, device=x.device) if mx0 is None else mx0.clone()
    _lib.call("llmc_observer_minmax_tensor_noalloc", C.c_void_p(_lib.ctx_for(x.device.index)), _lib.ptr(x),
              _lib.dtype_code(x.dtype), C.c_int64(x.shape[0]), C.c_int64(x.shape[1]), C.c_int64(x.stride(0)),
              _lib.ptr(mn), _lib.ptr(mx), accumulate)
    return mn, mx


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_noalloc_matches_workspace_observer_on_two_calls(dtype):
    g = torch.Generator(device="cuda").manual_seed(11)
    # First call: many rows, extremes planted mid-matrix.  Second call: fewer rows with a
    # narrower range, so row slots left over from the first call would change the answer.
    a = torch.randn(4096, 1000, device="cuda", generator=g).to(dtype)
    a[1234, 567] = 40.0
    a[3001, 3] = -37.5
    b = (0.25 * torch.randn(513, 777, device="cuda", generator=g)).to(dtype)
    ref_a, ref_b = _workspace_path(a, 0), _workspace_path(b, 0)
    got_a, got_b = _noalloc_path(a, 0), _noalloc_path(b, 0)
    torch.cuda.synchronize()
    for ref, got in ((ref_a, got_a), (ref_b, got_b)):
        torch.testing.assert_close(got[0], ref[0], rtol=0, atol=0)
        torch.testing.assert_close(got[1], ref[1], rtol=0, atol=0)
    assert float(got_a[1]) == 40.0 and float(got_a[0]) == -37.5
    assert float(got_b[1]) < 40.0


@pytest.mark.gpu
def test_noalloc_running_update_and_strided_view():
    g = torch.Generator(device="cuda").manual_seed(12)
    base = torch.randn(MAX_ROWS, 130, device="cuda", generator=g)
    x = base[:, 1:129]  # row stride 130, the full row limit
    mn0 = torch.tensor([-0.5], device="cuda")
    mx0 = torch.tensor([9.0], device="cuda")
    for _ in range(2):
        ref = _workspace_path(x, 1, mn0, mx0)
        got = _noalloc_path(x, 1, mn0, mx0)
        torch.cuda.synchronize()
        assert float(got[0]) == float(ref[0]) == float(x.min())
        assert float(got[1]) == float(ref[1]) == 9.0


@pytest.mark.gpu
def test_noalloc_call_allocates_no_device_memory():
    """The property the entry exists for.  On a fresh context (empty workspace) the calls after
    the first one leave the device's free memory unchanged, while the workspace observer on the
    same context has to grow its workspace (a cudaMalloc that shows in the free memory), which
    shows that the check would see an allocation.  The control input has 1 Mi rows, so that
    workspace (two floats a row, 8 MiB) is larger than the 2 MiB pages the driver hands out;
    a small cudaMalloc can be served from a page the context already holds."""
    lib = _lib.load()
    c = C.c_void_p()
    assert lib.llmc_init(0, C.byref(c)) == 0, _lib.last_error()
    try:
        assert lib.llmc_set_stream(c, C.c_void_p(torch.cuda.current_stream().cuda_stream or 1)) == 0
        x = torch.randn(8192, 1024, device="cuda")
        y = torch.randn(1 << 20, 4, device="cuda")  # control input for the workspace observer
        mn = torch.zeros(1, device="cuda")
        mx = torch.zeros(1, device="cuda")
        args = (_lib.ptr(x), _lib.dtype_code(x.dtype), C.c_int64(x.shape[0]), C.c_int64(x.shape[1]),
                C.c_int64(x.stride(0)))

        def noalloc():
            assert lib.llmc_observer_minmax_tensor_noalloc(c, *args, _lib.ptr(mn), _lib.ptr(mx), 0) == 0, \
                _lib.last_error()

        noalloc()  # first call on the context's device: address lookup
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            noalloc()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0
        assert float(mn) == float(x.min()) and float(mx) == float(x.max())
        st = lib.llmc_observer_minmax(c, _lib.ptr(y), _lib.dtype_code(y.dtype), C.c_int64(y.shape[0]),
                                      C.c_int64(y.shape[1]), C.c_int64(y.stride(0)), _lib.STRATEGY["tensor"],
                                      C.c_int64(y.shape[1]), _lib.ptr(mn), _lib.ptr(mx), 0)
        assert st == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] < free0
        assert float(mn) == float(y.min()) and float(mx) == float(y.max())
    finally:
        lib.llmc_destroy(c)


@pytest.mark.gpu
def test_noalloc_rejects_rows_over_the_limit():
    x = torch.zeros(MAX_ROWS + 1, 8, device="cuda")
    launches = _lib.launch_count(0)
    with pytest.raises(LlmcError, match="static row buffer"):
        _noalloc_path(x, 0)
    assert _lib.launch_count(0) == launches
