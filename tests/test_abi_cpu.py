"""CPU-side checks of the C ABI library: it builds, loads without a GPU, and exports exactly
what include/llmc_b200.h declares.  No compute calls (there is no GPU here)."""

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llmc_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(llmc_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib_path():
    from llmcompressorsharp_b200 import build

    return build.build()


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("llmc_init", "llmc_hessian_update", "llmc_chol_inverse", "llmc_gptq_quantize",
                 "llmc_rtn_quantize", "llmc_observer_minmax", "llmc_act_absmax", "llmc_smooth_apply",
                 "llmc_sparsegpt_prune", "llmc_awq_search", "llmc_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    lib = ctypes.CDLL(lib_path)
    for n in declared_functions():
        assert getattr(lib, n) is not None


def test_ctypes_signatures_cover_header(lib_path):
    from llmcompressorsharp_b200 import _lib

    assert sorted(_lib.exported_symbols()) == declared_functions()
    lib = _lib.load(lib_path)
    assert lib.llmc_abi_version() == 1


def test_qconfig_layout_matches_header():
    from llmcompressorsharp_b200 import _lib

    src = open(HEADER).read()
    body = src[src.index("typedef struct {"):src.index("} llmc_qconfig;")]
    fields = re.findall(r"(int32_t|float)\s+(\w+);", body)
    assert [f for _, f in fields] == [n for n, _ in _lib.QConfig._fields_]
    assert ctypes.sizeof(_lib.QConfig) == 4 * len(fields)


def test_no_gpu_call_fails_cleanly(lib_path):
    """Without a GPU, llmc_init returns an error status with a message (no abort)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from llmcompressorsharp_b200 import _lib

    lib = _lib.load(lib_path)
    out = ctypes.c_void_p()
    st = lib.llmc_init(0, ctypes.byref(out))
    assert st != 0 and out.value is None
    assert _lib.last_error()


def test_null_arguments_map_to_statuses(lib_path):
    from llmcompressorsharp_b200 import _lib

    lib = _lib.load(lib_path)
    assert lib.llmc_init(0, None) == 1  # LLMC_ERR_INVALID_ARG
    assert lib.llmc_hessian_update(None, None, 0, 1, 1) == 1
    assert lib.llmc_gptq_quantize(None, None, 0, 1, 1, 1, None, 1, None, None, 1, None, None, None) == 1


def test_error_mapping():
    from llmcompressorsharp_b200 import errors

    with pytest.raises(ValueError):
        errors.raise_for_status(1, "x")
    with pytest.raises(NotImplementedError):
        errors.raise_for_status(3, "x")
    with pytest.raises(errors.ArgumentOutOfRangeError):
        errors.raise_for_status(10, "x")
    with pytest.raises(errors.NotPositiveDefiniteError):
        errors.raise_for_status(4, "x")


def test_nccl_unique_id_through_the_abi():
    """NCCL is opened at the first collective call (no link dependency); a unique id needs no
    GPU, and a short buffer is rejected before NCCL is touched."""
    import ctypes as C

    from llmcompressorsharp_b200 import _lib

    lib = _lib.load()
    short = (C.c_uint8 * 64)()
    assert lib.llmc_nccl_unique_id(C.cast(short, C.c_void_p), 64) == 2  # LLMC_ERR_SHAPE
    assert "need 128" in _lib.last_error()
    buf = (C.c_uint8 * _lib.NCCL_UNIQUE_ID_BYTES)()
    st = lib.llmc_nccl_unique_id(C.cast(buf, C.c_void_p), len(buf))
    if st == 3:  # LLMC_ERR_UNSUPPORTED: no libnccl.so.2 on this host
        pytest.skip(_lib.last_error())
    assert st == 0, _lib.last_error()
    assert any(bytes(buf))
    assert lib.llmc_nccl_comm_destroy(None) == 0
