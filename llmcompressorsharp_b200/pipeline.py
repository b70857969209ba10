"""Layer-level GPTQ pipeline: the one-shot flow of GPTQModifier.OnStart/OnEnd
(src/LLMCompressorSharp.Core/Algorithms/Gptq/GPTQModifier.cs:59-137) for a stack of decoder
layers whose calibration activations are given per input site.

One Hessian per distinct input site (q/k/v share the attention input, gate/up the MLP
input); every weight that reads a site is quantised against that site's factor U.  The
result per weight is the packed int codes, scales and zero-points (plus, optionally, the
fp32 fake-quantised weight the reference returns).

Multi-GPU: calibration tokens are split across ranks; each rank accumulates its partial
H for every site, the partial Hessians are summed onto the layer's owner rank
(``torch.distributed.reduce`` over NCCL), and owners solve their layers (layers are dealt
round-robin).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .gptq import GPTQConfig, param_shape


@dataclass
class SiteSpec:
    name: str
    d: int
    weights: list  # [(weight_name, out_features)]


def llama_sites(hidden: int, intermediate: int, n_heads: int, n_kv: int):
    head = hidden // n_heads
    kv = n_kv * head
    return [
        SiteSpec("attn_in", hidden, [("q_proj", hidden), ("k_proj", kv), ("v_proj", kv)]),
        SiteSpec("o_in", hidden, [("o_proj", hidden)]),
        SiteSpec("mlp_in", hidden, [("gate_proj", intermediate), ("up_proj", intermediate)]),
        SiteSpec("down_in", intermediate, [("down_proj", hidden)]),
    ]


class GptqPipeline:
    """Device-resident GPTQ over layers.  ``weights[l][name]`` are [out, in] device tensors,
    ``acts[site]`` are [T, d] device tensors (this rank's calibration tokens)."""

    def __init__(self, sites, cfg: GPTQConfig, device: torch.device, chunk_rows: int = 65536, keep_wq: bool = False):
        self.sites = sites
        self.cfg = cfg
        self.device = device
        self.chunk = chunk_rows
        self.keep_wq = keep_wq
        self.c = C.c_void_p(_lib.ctx_for(device.index))
        self.qc = cfg.to_c()
        maxd = max(s.d for s in sites)
        # one Hessian handle per site, reused layer after layer
        self.h = {}
        for s in sites:
            p = C.c_void_p()
            _lib.call("llmc_hessian_create", self.c, C.c_int64(s.d), C.byref(p))
            self.h[s.name] = p.value
        self.u = torch.empty(maxd * maxd, dtype=torch.float32, device=device)
        maxm = max(m for s in sites for _, m in s.weights)
        self.work = torch.empty(maxm * maxd, dtype=torch.float32, device=device)

    def close(self):
        for p in self.h.values():
            _lib.call("llmc_hessian_destroy", C.c_void_p(p))
        self.h = {}

    def hessian_ptr(self, site: str) -> int:
        p = C.c_void_p()
        _lib.call("llmc_hessian_data", C.c_void_p(self.h[site]), C.byref(p))
        return p.value

    def accumulate(self, site: SiteSpec, x: torch.Tensor, out_h: torch.Tensor | None = None):
        """H_site = sum over chunks of X^T X (reset first).  Optionally copy H out."""
        _lib.ctx_for(self.device.index)
        h = C.c_void_p(self.h[site.name])
        _lib.call("llmc_hessian_reset", h)
        T = x.shape[0]
        for r0 in range(0, T, self.chunk):
            r1 = min(T, r0 + self.chunk)
            _lib.call("llmc_hessian_update", h, C.c_void_p(x.data_ptr() + r0 * x.stride(0) * x.element_size()),
                      _lib.dtype_code(x.dtype), C.c_int64(r1 - r0), C.c_int64(x.stride(0)))
        if out_h is not None:
            out_h.copy_(torch.as_tensor(_HView(self.hessian_ptr(site.name), site.d), device=self.device))

    def solve_site(self, site: SiteSpec, h_ptr: int, weights: dict, outputs: dict):
        """U from the site's H (upper triangle), then GPTQ of each weight reading the site."""
        d = site.d
        _lib.ctx_for(self.device.index)
        _lib.call("llmc_chol_inverse", self.c, C.c_void_p(h_ptr), C.c_int64(d), C.c_int64(d),
                  C.c_float(self.cfg.dampening_frac), 1, _lib.ptr(self.u), C.c_int64(d), 1)
        for wname, m in site.weights:
            w = weights[wname]
            out = outputs[wname]
            wq = out.get("wq")
            if wq is None:
                wq = self.work[: m * d].view(m, d)
            _lib.call("llmc_gptq_quantize", self.c, _lib.ptr(w), _lib.dtype_code(w.dtype), C.c_int64(m), C.c_int64(d),
                      C.c_int64(w.stride(0)), _lib.ptr(self.u), C.c_int64(d), C.byref(self.qc), _lib.ptr(wq),
                      C.c_int64(d), _lib.ptr(out["codes"]), _lib.ptr(out["scales"]), _lib.ptr(out["zero_points"]))

    def alloc_outputs(self, layer_weights: dict):
        outs = {}
        for s in self.sites:
            for wname, m in s.weights:
                n = s.d
                shp = param_shape(self.cfg.strategy, m, n, self.cfg.group_size)
                outs[wname] = {
                    "codes": torch.empty(m, (n + 1) // 2 if self.cfg.num_bits <= 4 else n, dtype=torch.uint8,
                                         device=self.device),
                    "scales": torch.empty(shp, dtype=torch.float32, device=self.device),
                    "zero_points": torch.empty(shp, dtype=torch.int32, device=self.device),
                }
                if self.keep_wq:
                    outs[wname]["wq"] = torch.empty(m, n, dtype=torch.float32, device=self.device)
        return outs

    def run_layer(self, acts: dict, weights: dict, outputs: dict):
        for s in self.sites:
            self.accumulate(s, acts[s.name])
            self.solve_site(s, self.hessian_ptr(s.name), weights, outputs)


class _HView:
    def __init__(self, ptr, d):
        self.__cuda_array_interface__ = {"shape": (d, d), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}
