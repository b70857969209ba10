"""ctypes binding of libllmc_b200.so (the C ABI in include/llmc_b200.h).

There is no fallback: if the shared library is missing or cannot find a B200, every call
raises.  Device tensors are passed as raw pointers; the library runs on the current
torch CUDA stream of the tensor's device so that its kernels are ordered with torch's
own allocations and copies.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

from .errors import raise_for_status

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllmc_b200.so")

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
STRATEGY = {"tensor": 0, "channel": 1, "token": 2, "group": 3}
CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy


class QConfig(C.Structure):
    """llmc_qconfig."""

    _fields_ = [
        ("num_bits", C.c_int32),
        ("symmetric", C.c_int32),
        ("strategy", C.c_int32),
        ("channel_axis", C.c_int32),
        ("group_size", C.c_int32),
        ("block_size", C.c_int32),
        ("damp", C.c_float),
        ("act_order", C.c_int32),
        ("sparsity", C.c_float),
        ("mask_n", C.c_int32),
        ("mask_m", C.c_int32),
    ]


P = C.c_void_p
I32, I64, F32 = C.c_int32, C.c_int64, C.c_float

# name -> argtypes (every function returns llmc_status as int32)
NCCL_UNIQUE_ID_BYTES = 128  # LLMC_NCCL_UNIQUE_ID_BYTES

_SIGS = {
    "llmc_abi_version": [],
    "llmc_init": [I32, C.POINTER(P)],
    "llmc_destroy": [P],
    "llmc_set_stream": [P, P],
    "llmc_set_sm_limit": [P, I32],
    "llmc_set_wait_limit": [P, I64],
    "llmc_set_deferred_errors": [P, I32],
    "llmc_sync": [P],
    "llmc_launch_count": [P, C.POINTER(I64)],
    "llmc_hessian_create": [P, I64, C.POINTER(P)],
    "llmc_hessian_update": [P, P, I32, I64, I64],
    "llmc_hessian_get": [P, P],
    "llmc_hessian_data": [P, C.POINTER(P)],
    "llmc_hessian_reset": [P],
    "llmc_hessian_sample_count": [P, C.POINTER(I64)],
    "llmc_hessian_add_samples": [P, I64],
    "llmc_hessian_destroy": [P],
    "llmc_nccl_unique_id": [P, I64],
    "llmc_nccl_comm_init": [P, I32, I32, P, I64, C.POINTER(P)],
    "llmc_nccl_comm_destroy": [P],
    "llmc_hessian_allreduce": [P, P],
    "llmc_hessian_reduce": [P, P, I32],
    "llmc_chol_inverse": [P, P, I64, I64, F32, I32, P, I64, I32],
    "llmc_upper_factor": [P, P, I64, I64, P, I64],
    "llmc_gptq_quantize": [P, P, I32, I64, I64, I64, P, I64, C.POINTER(QConfig), P, I64, P, P, P],
    "llmc_gptq_quantize_batch": [P, I32, P, P, P, I32, I64, P, I64, C.POINTER(QConfig), P, I64, P, P, P],
    "llmc_gptq_act_order_perm": [P, P, I64, I64, P],
    "llmc_permute_hessian": [P, P, I64, I64, I32, P, P, I64],
    "llmc_gptq_quantize_batch_perm": [P, I32, P, P, P, I32, I64, P, I64, P, C.POINTER(QConfig), P, I64, P, P, P],
    "llmc_sparsegpt_prune": [P, P, I32, I64, I64, I64, P, I64, C.POINTER(QConfig), P, I64, P],
    "llmc_observer_minmax": [P, P, I32, I64, I64, I64, I32, I64, P, P, I32],
    "llmc_observer_minmax_tensor_noalloc": [P, P, I32, I64, I64, I64, P, P, I32],
    "llmc_affine_params": [P, P, P, I64, I32, I32, P, P],
    "llmc_observer_mse": [P, P, I32, I64, I32, I32, I32, C.POINTER(F32), C.POINTER(I32), P],
    "llmc_fake_quantize": [P, P, I32, I64, F32, I32, I32, I32, P, P],
    "llmc_rtn_quantize": [P, P, I32, I64, I64, I64, C.POINTER(QConfig), P, P, P, P],
    "llmc_int4_pack": [P, P, I64, I32, P],
    "llmc_int4_unpack_dequant": [P, P, I64, F32, I32, I32, P],
    "llmc_pack_compressed_tensors": [P, P, I64, I64, I64, P, I32, I64, I32, I32, P, I64, P],
    "llmc_act_quant_per_token": [P, P, I32, I64, I64, I64, I32, I32, P, I64, P, P, P, I64],
    "llmc_act_absmax": [P, P, I32, I64, I64, I64, P, I32],
    "llmc_smooth_apply": [P, P, P, I32, P, I32, I64, I64, F32, P],
    "llmc_scale_apply": [P, P, P, I32, P, I32, I64, I64],
    "llmc_awq_search": [P, P, I32, I64, I64, I64, P, I32, C.POINTER(QConfig), P, P, P],
}

_lib = None
_lock = threading.Lock()
_ctxs: dict[int, int] = {}


def exported_symbols() -> list[str]:
    return ["llmc_last_error"] + list(_SIGS)


def load(path: str | None = None) -> C.CDLL:
    """Load the shared library (no GPU needed).  Raises if it was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"libllmc_b200.so not found at {p}; build it with `python -m llmcompressorsharp_b200.build` "
                "(the CUDA library is required: there is no CPU implementation)")
        lib = C.CDLL(p)
        lib.llmc_last_error.restype = C.c_char_p
        lib.llmc_last_error.argtypes = []
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = C.c_int32
        _lib = lib
        return lib


def last_error() -> str:
    return load().llmc_last_error().decode("utf-8", "replace")


def call(name: str, *args) -> None:
    lib = load()
    st = getattr(lib, name)(*args)
    if st != 0:
        raise_for_status(st, f"{name}: {last_error()}")


def ctx_for(device_index: int) -> int:
    """Per-device context handle (created on first use), bound to torch's current stream."""
    import torch

    lib = load()
    h = _ctxs.get(device_index)
    if h is None:
        with _lock:
            h = _ctxs.get(device_index)
            if h is None:
                out = P()
                st = lib.llmc_init(device_index, C.byref(out))
                if st != 0:
                    raise_for_status(st, f"llmc_init: {last_error()}")
                h = out.value
                _ctxs[device_index] = h
    # torch reports the legacy default stream as handle 0; pass it as cudaStreamLegacy
    # (0x1) so the library's kernels are ordered with torch's work on that stream.
    stream = torch.cuda.current_stream(device_index).cuda_stream or CUDA_STREAM_LEGACY
    st = lib.llmc_set_stream(h, P(stream))
    if st != 0:
        raise_for_status(st, f"llmc_set_stream: {last_error()}")
    return h


def launch_count(device_index: int = 0) -> int:
    v = I64()
    call("llmc_launch_count", P(ctx_for(device_index)), C.byref(v))
    return int(v.value)


def dtype_code(dt) -> int:
    import torch

    if dt == torch.float32:
        return DTYPE_F32
    if dt == torch.bfloat16:
        return DTYPE_BF16
    if dt == torch.float16:
        return DTYPE_F16
    raise TypeError(f"unsupported dtype {dt}")


def ptr(t) -> P:
    return P(t.data_ptr()) if t is not None else P(0)
