"""llmc_set_deferred_errors: the factorisation decides a non-positive-definite input on the
device and reports it at the next llmc_sync, with the same outputs as the synchronous path.

HessianInverseSolver.cs:85-91 (pinv fallback; pinv of the zero matrix is zero) and
GptqBlockQuantizer.cs:112-118 (U = Hinv when chol(Hinv) fails)."""

import ctypes as C

import pytest
import torch

from llmcompressorsharp_b200 import _lib
from oracle import hessian as o_hess

pytestmark = pytest.mark.gpu
NOT_PD = 4


def _ctx(deferred):
    lib = _lib.load()
    c = C.c_void_p()
    assert lib.llmc_init(0, C.byref(c)) == 0, _lib.last_error()
    assert lib.llmc_set_stream(c, C.c_void_p(torch.cuda.current_stream().cuda_stream or 1)) == 0
    assert lib.llmc_set_deferred_errors(c, deferred) == 0
    return lib, c


def _upper(lib, c, h, damp=0.01, upper_only=1):
    d = h.shape[0]
    out = torch.full((d, d), 7.0, device="cuda")
    st = lib.llmc_chol_inverse(c, _lib.ptr(h), d, d, C.c_float(damp), upper_only, _lib.ptr(out), d, 1)
    return st, out


def _spd(d, seed):
    x = torch.randn(4 * d, d, generator=torch.Generator().manual_seed(seed))
    return x.t() @ x


@pytest.mark.parametrize("d", [200, 640])
def test_deferred_factor_equals_synchronous(d):
    h = _spd(d, d).cuda()
    lib, cs = _ctx(0)
    lib2, cd = _ctx(1)
    try:
        st, u_sync = _upper(lib, cs, h)
        assert st == 0, _lib.last_error()
        st, u_def = _upper(lib2, cd, h)
        assert st == 0, _lib.last_error()
        assert lib2.llmc_sync(cd) == 0
        torch.cuda.synchronize()
        assert torch.equal(u_sync, u_def)
        want = o_hess.upper_factor(o_hess.hessian_inverse(h.cpu(), 0.01))
        assert float((u_def.cpu() - want).norm() / want.norm()) < 1e-4
    finally:
        lib.llmc_destroy(cs)
        lib2.llmc_destroy(cd)


def test_deferred_zero_matrix_gives_zero_factor_without_error():
    lib, c = _ctx(1)
    try:
        h = torch.zeros(300, 300, device="cuda")
        st, u = _upper(lib, c, h, damp=0.0)
        assert st == 0
        assert lib.llmc_sync(c) == 0
        assert torch.count_nonzero(u) == 0
    finally:
        lib.llmc_destroy(c)


def test_deferred_non_pd_reported_at_sync_and_cleared():
    lib, c = _ctx(1)
    try:
        h = -torch.eye(256, device="cuda")
        st, u = _upper(lib, c, h, damp=0.0)
        assert st == 0  # nothing was read back: the call only enqueued the work
        assert lib.llmc_sync(c) == NOT_PD
        assert "not positive definite" in _lib.last_error()
        assert torch.count_nonzero(u) == 0
        assert lib.llmc_sync(c) == 0  # the word was cleared
        # the synchronous path takes the pinv fallback instead: pinv(-I) = -I, which has no
        # Cholesky factor, so U = Hinv (HessianInverseSolver.cs:85-91, GptqBlockQuantizer.cs:112-118)
        assert lib.llmc_set_deferred_errors(c, 0) == 0
        st, u = _upper(lib, c, h, damp=0.0)
        assert st == 0, _lib.last_error()
        assert float((u + torch.eye(256, device="cuda")).abs().max()) < 1e-5
    finally:
        lib.llmc_destroy(c)


def test_deferred_upper_factor_falls_back_to_hinv():
    lib, c = _ctx(1)
    try:
        d = 192
        hinv = torch.eye(d, device="cuda")
        hinv[5, 5] = -1.0  # chol(Hinv) fails -> U = Hinv (GptqBlockQuantizer.cs:112-118)
        out = torch.empty(d, d, device="cuda")
        assert lib.llmc_upper_factor(c, _lib.ptr(hinv), d, d, _lib.ptr(out), d) == 0
        assert lib.llmc_sync(c) == 0
        assert torch.equal(out, hinv)
        good = torch.linalg.inv(_spd(d, 3)).cuda()
        good = 0.5 * (good + good.t())
        assert lib.llmc_upper_factor(c, _lib.ptr(good), d, d, _lib.ptr(out), d) == 0
        assert lib.llmc_sync(c) == 0
        want = o_hess.upper_factor(good.cpu())
        assert float((out.cpu() - want).norm() / want.norm()) < 1e-4
    finally:
        lib.llmc_destroy(c)
