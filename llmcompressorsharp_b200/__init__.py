"""llmcompressorsharp_b200 — LLMCompressorSharp's one-shot compression hot path on B200.

Calibration Hessian accumulation, the damped Cholesky inverse, the GPTQ / SparseGPT
column-block solve, min-max observers with RTN int4/int8 packing, SmoothQuant and AWQ
scale search run as sm_100a CUDA kernels in ``libllmc_b200.so`` behind the C ABI declared
in ``include/llmc_b200.h``.  This package is the Python mirror of the reference's
primitive and modifier API on top of that ABI (ctypes; torch only supplies device memory
and streams).
"""

from .errors import (ArgumentError, ArgumentOutOfRangeError, CudaError, InvalidOperationError, LlmcError,
                     NotPositiveDefiniteError, NotSupportedError, ShapeError)
from .hessian import ActivationHookManager, HessianAccumulator, HessianInverseSolver, upper_factor
from .quantization import (FakeQuantize, GroupMinMaxObserver, Int4PackedTensor, MinMaxObserver,
                           MovingAverageMinMaxObserver, MSEObserver, PerChannelMinMaxObserver, affine_params,
                           quantize_per_token)
from .gptq import (GPTQConfig, GPTQModifier, GptqBlockQuantizer, GptqResult, act_order_perm, gptq_quantize_act_order,
                   gptq_quantize_u)
from .rtn import RtnConfig, RtnModifier, rtn_quantize
from .smoothquant import SmoothQuantConfig, SmoothQuantMapping, SmoothQuantModifier, act_absmax, smooth_apply
from .sparsegpt import SparseGPTConfig, SparseGPTModifier, sparsegpt_prune_u
from .awq import AWQConfig, AWQModifier, awq_search, scale_apply
from .session import (CompressionSession, CompressionState, ModifierBase, ModifierLifecycleError, SessionStatus,
                      TargetMatcher)
from .output import CompressedTensorsWriter, SafetensorsWriter

__all__ = [n for n in dir() if not n.startswith("_")]
