"""GPTQ on the B200: config, block quantiser and modifier.

Mirrors ``GPTQConfig`` (src/LLMCompressorSharp.Core/Algorithms/Configs/GPTQConfig.cs:22-59),
``GptqBlockQuantizer`` (Algorithms/Gptq/GptqBlockQuantizer.cs:46-275) and ``GPTQModifier``
(Algorithms/Gptq/GPTQModifier.cs:28-156).  Adds ``group_size`` for the group strategy.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._device import ctx, supported_dtype, target_device, to_device
from .errors import ArgumentError, InvalidOperationError, NotPositiveDefiniteError, NotSupportedError
from .hessian import ActivationHookManager, HessianAccumulator, HessianInverseSolver, upper_factor
from .session import CompressionState, ModifierBase

_ACT_ORDER_MSG = ("GPTQConfig.ActOrder=true is not yet implemented. "
                  "Column reordering by Hessian diagonal is deferred to a future release.")


@dataclass
class GPTQConfig:
    """GPTQConfig.cs:22-59 (same defaults) + group_size."""

    num_bits: int = 4
    symmetric: bool = True
    strategy: str = "channel"
    channel_axis: int = 0
    block_size: int = 128
    dampening_frac: float = 0.01
    act_order: bool = False
    group_size: int = 128
    targets: list = field(default_factory=list)
    ignore: list = field(default_factory=list)
    type: str = "GPTQ"

    def to_c(self) -> _lib.QConfig:
        if self.strategy not in _lib.STRATEGY:
            raise NotSupportedError(f"Quantization strategy '{self.strategy}' is not supported by GptqBlockQuantizer.")
        return _lib.QConfig(num_bits=self.num_bits, symmetric=int(self.symmetric),
                            strategy=_lib.STRATEGY[self.strategy], channel_axis=self.channel_axis,
                            group_size=self.group_size, block_size=self.block_size, damp=self.dampening_frac,
                            act_order=int(self.act_order), sparsity=0.0, mask_n=0, mask_m=0)


@dataclass
class GptqResult:
    wq: torch.Tensor            # fp32 fake-quantised weight [m, n]
    codes: torch.Tensor | None  # uint8 codes (packed two per byte for num_bits <= 4)
    scales: torch.Tensor        # fp32 [1] / [m] / [m, G]
    zero_points: torch.Tensor   # int32, same shape


def param_shape(strategy: str, m: int, n: int, group_size: int):
    if strategy == "tensor":
        return (1,)
    if strategy == "channel":
        return (m,)
    return (m, (n + group_size - 1) // group_size)


def gptq_quantize_u(weight: torch.Tensor, upper: torch.Tensor, config: GPTQConfig, want_codes: bool = True,
                    out: torch.Tensor | None = None) -> GptqResult:
    """Column loop of GptqBlockQuantizer.Quantize (:122-181) given the upper factor U.
    Runs on the weight's CUDA device (host tensors are staged)."""
    if weight is None or upper is None or config is None:
        raise ArgumentError("weight, hinv and config must not be null")
    if config.act_order:
        raise NotSupportedError(_ACT_ORDER_MSG)
    dev = target_device(weight, upper)
    w = to_device(supported_dtype(weight.detach()), dev)
    u = to_device(upper.detach(), dev, torch.float32)
    m, n = w.shape
    wq = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=dev)
    codes = None
    if want_codes and config.num_bits <= 8:
        codes = torch.empty(m, (n + 1) // 2 if config.num_bits <= 4 else n, dtype=torch.uint8, device=dev)
    shp = param_shape(config.strategy, m, n, config.group_size)
    scales = torch.empty(shp, dtype=torch.float32, device=dev)
    zps = torch.empty(shp, dtype=torch.int32, device=dev)
    cfg = config.to_c()
    _lib.call("llmc_gptq_quantize", C.c_void_p(ctx(dev)), _lib.ptr(w), _lib.dtype_code(w.dtype), C.c_int64(m),
              C.c_int64(n), C.c_int64(n), _lib.ptr(u), C.c_int64(n), C.byref(cfg), _lib.ptr(wq), C.c_int64(wq.stride(0)),
              _lib.ptr(codes), _lib.ptr(scales), _lib.ptr(zps))
    return GptqResult(wq, codes, scales, zps)


def act_order_perm(h: torch.Tensor, upper_only: bool = False) -> torch.Tensor:
    """Extension (the reference rejects ActOrder, GPTQModifier.cs:47-56): the GPTQ activation
    order of a Hessian, columns by decreasing H[k][k] (equal values by index, NaN first), as an
    int32 device tensor.  ``upper_only`` is accepted for symmetry with the other calls; only the
    diagonal is read."""
    dev = target_device(h)
    hd = to_device(h.detach(), dev, torch.float32)
    d = hd.shape[0]
    perm = torch.empty(d, dtype=torch.int32, device=dev)
    _lib.call("llmc_gptq_act_order_perm", C.c_void_p(ctx(dev)), _lib.ptr(hd), C.c_int64(d), C.c_int64(hd.stride(0)),
              _lib.ptr(perm))
    return perm


def gptq_quantize_act_order(weight: torch.Tensor, h: torch.Tensor, config: GPTQConfig, want_codes: bool = True,
                            upper_only: bool = False) -> tuple[GptqResult, torch.Tensor]:
    """Extension: GPTQ with activation order and static groups, from the Hessian H (not Hinv:
    the order needs diag(H)).  perm = act_order_perm(H); U_p = the factor of H[perm][:, perm]
    damped by ``config.dampening_frac`` (HessianInverseSolver.cs:44-92); scales and zero-points
    from the original weight per original column group (GptqBlockQuantizer.cs:97); the column
    loop over W[:, perm]; outputs in the original column order.  Returns (result, perm)."""
    if weight is None or h is None or config is None:
        raise ArgumentError("weight, hessian and config must not be null")
    dev = target_device(weight, h)
    w = to_device(supported_dtype(weight.detach()), dev)
    hd = to_device(h.detach(), dev, torch.float32)
    m, n = w.shape
    if hd.shape != (n, n):
        raise ArgumentError("Hessian must be a square 2-D tensor matching the weight's in_features.")
    perm = act_order_perm(hd)
    c = C.c_void_p(ctx(dev))
    hp = torch.empty(n, n, dtype=torch.float32, device=dev)
    _lib.call("llmc_permute_hessian", c, _lib.ptr(hd), C.c_int64(n), C.c_int64(hd.stride(0)), C.c_int32(int(upper_only)),
              _lib.ptr(perm), _lib.ptr(hp), C.c_int64(n))
    up = HessianInverseSolver.upper(hp, config.dampening_frac)
    wq = torch.empty(m, n, dtype=torch.float32, device=dev)
    codes = None
    if want_codes and config.num_bits <= 8:
        codes = torch.empty(m, (n + 1) // 2 if config.num_bits <= 4 else n, dtype=torch.uint8, device=dev)
    shp = param_shape(config.strategy, m, n, config.group_size)
    scales = torch.empty(shp, dtype=torch.float32, device=dev)
    zps = torch.empty(shp, dtype=torch.int32, device=dev)
    cfg = config.to_c()
    wp = (C.c_void_p * 1)(w.data_ptr())
    mp = (C.c_int64 * 1)(m)
    lp = (C.c_int64 * 1)(w.stride(0))
    _lib.call("llmc_gptq_quantize_batch_perm", c, C.c_int32(1), wp, mp, lp, _lib.dtype_code(w.dtype), C.c_int64(n),
              _lib.ptr(up), C.c_int64(n), _lib.ptr(perm), C.byref(cfg), _lib.ptr(wq), C.c_int64(n), _lib.ptr(codes),
              _lib.ptr(scales), _lib.ptr(zps))
    return GptqResult(wq, codes, scales, zps), perm


class GptqBlockQuantizer:
    """GptqBlockQuantizer (GptqBlockQuantizer.cs:46-275)."""

    @staticmethod
    def quantize(weight: torch.Tensor, hinv: torch.Tensor, config: GPTQConfig) -> torch.Tensor:
        """Quantize(W, Hinv, cfg) (:71-190): U = chol(Hinv)^T (Hinv fallback), then the
        column loop; returns the fp32 fake-quantised weight on W's device."""
        if weight is None or hinv is None or config is None:
            raise ArgumentError("weight, hinv and config must not be null")
        if config.act_order:
            raise NotSupportedError(_ACT_ORDER_MSG)
        res = GptqBlockQuantizer.quantize_full(weight, hinv, config)
        return res.wq if weight.is_cuda else res.wq.cpu()

    @staticmethod
    def quantize_full(weight, hinv, config) -> GptqResult:
        dev = target_device(weight, hinv)
        return gptq_quantize_u(weight, upper_factor(to_device(hinv.detach(), dev, torch.float32)), config)


class GPTQModifier(ModifierBase):
    """GPTQModifier.cs:28-156: hooks accumulate H per targeted Linear during calibration;
    OnEnd factors each H on the device and quantises the weight.

    ``share_inputs=True`` lets modules that receive the very same input tensor in a forward
    pass (q/k/v, gate/up) share one accumulator — the results are identical to one
    accumulator per weight, with the repeated X^T X products skipped.
    """

    def __init__(self, config: GPTQConfig, share_inputs: bool = False):
        if config is None:
            raise ArgumentError("config must not be null")
        super().__init__("GPTQ", config.targets, config.ignore)
        self.config = config
        self.share_inputs = share_inputs
        self._hooks: ActivationHookManager | None = None
        self._acc: dict[str, HessianAccumulator] | None = None
        self._alias: dict[int, HessianAccumulator] = {}

    def on_initialize(self, state):
        if self.config.act_order:  # GPTQModifier.cs:47-56
            raise NotSupportedError(_ACT_ORDER_MSG)

    def on_start_core(self, state: CompressionState):
        if state.named_modules is None:  # :61-66
            raise InvalidOperationError(
                "GPTQModifier requires CompressionState.NamedModules to be populated. "
                "Set it to the named Linear modules before calling OnStart.")
        self._hooks = ActivationHookManager()
        self._acc = {}
        self._alias = {}
        owners: dict[tuple, tuple] = {}  # key -> (accumulator, the input it saw)
        for wname in self.targeted_names(state):
            lname = wname[: -len(".weight")] if wname.endswith(".weight") else wname
            module = state.named_modules.get(lname)
            if module is None:  # :79-85
                continue
            in_features = state.named_weights[wname].shape[-1]
            dev = target_device(state.named_weights[wname])
            acc = HessianAccumulator(in_features, dev)
            self._acc[wname] = acc
            if self.share_inputs:
                self._register_shared(module, acc, owners)
            else:
                self._hooks.register_for(module, acc)

    def _register_shared(self, module, acc, owners):
        """Hook that updates ``acc`` unless the module's input is the same tensor another
        shared module already accumulated in this forward pass; then ``acc`` aliases it."""
        from .hessian import ForwardHookHandle

        alias = self._alias

        def hook(mod, inputs, output):
            x = inputs[0]
            # Same tensor = same address, shape, strides, dtype and in-place version.  The entry
            # holds x itself: while it stands, the caching allocator cannot give x's memory to
            # a later tensor (say the next norm's output after x was freed), which would
            # otherwise match the key with different data.
            key = (x.data_ptr(), tuple(x.shape), tuple(x.stride()), x.dtype, x._version)
            entry = owners.get(key)
            owner = entry[0] if entry is not None else None
            if owner is None:
                if id(acc) in alias:
                    raise InvalidOperationError("GPTQ share_inputs: a module that shared its input earlier "
                                                "received a different input")
                owners.clear()
                owners[key] = (acc, x)
                acc.update(x)
            elif owner is not acc:
                prev = alias.get(id(acc))
                if prev is not None and prev is not owner:
                    raise InvalidOperationError("GPTQ share_inputs: inconsistent input sharing between modules")
                alias[id(acc)] = owner
            return output

        self._hooks._handles.append(ForwardHookHandle(module.register_forward_hook(hook)))

    def on_end_core(self, state: CompressionState):
        if self._hooks is not None:
            self._hooks.dispose()
            self._hooks = None
        if not self._acc:
            return
        alias = self._alias
        # Factor every distinct Hessian first, with the device context's errors deferred: the
        # factorisations are enqueued back to back (none reads a flag back to the host), and one
        # llmc_sync per device then reports whether any Hessian had no Cholesky factor.  Those
        # devices factor their Hessians again synchronously, which takes the reference's
        # pseudo-inverse fallback (HessianInverseSolver.cs:85-91); every weight is replaced only
        # after all factors exist.
        ucache: dict[int, torch.Tensor] = {}
        srcs = {}
        for acc in self._acc.values():
            src = alias.get(id(acc), acc)
            srcs.setdefault(id(src), src)
        by_dev: dict = {}
        for key, src in srcs.items():
            by_dev.setdefault(src.raw().device, []).append((key, src))
        for dev, items in by_dev.items():
            c = C.c_void_p(ctx(dev))
            _lib.call("llmc_set_deferred_errors", c, C.c_int32(1))
            redo = False
            try:
                with torch.cuda.device(dev):
                    for key, src in items:
                        ucache[key] = HessianInverseSolver.upper(src.raw(), self.config.dampening_frac, upper_only=True)
                _lib.call("llmc_sync", c)
            except NotPositiveDefiniteError:
                redo = True
            finally:
                _lib.call("llmc_set_deferred_errors", c, C.c_int32(0))
            if redo:
                with torch.cuda.device(dev):
                    for key, src in items:
                        ucache[key] = HessianInverseSolver.upper(src.raw(), self.config.dampening_frac, upper_only=True)
        for wname, acc in self._acc.items():
            key = id(alias.get(id(acc), acc))
            w = state.named_weights[wname]
            res = gptq_quantize_u(w, ucache[key], self.config)
            state.named_weights[wname] = res.wq if w.is_cuda else res.wq.cpu()
            state.compressed[wname] = {"codes": res.codes, "scales": res.scales, "zero_points": res.zero_points,
                                       "num_bits": self.config.num_bits, "symmetric": self.config.symmetric,
                                       "strategy": self.config.strategy, "group_size": self.config.group_size}

    def on_finalize_core(self, state):
        if self._hooks is not None:
            self._hooks.dispose()
            self._hooks = None
        if self._acc is not None:
            for a in self._acc.values():
                a.dispose()
            self._acc = None
