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
        # fp32 working copy of the largest stacked solve (rows of all weights of one site)
        self.work = torch.empty(max(sum(m for _, m in s.weights) * s.d for s in sites), dtype=torch.float32,
                                device=device)

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
        """U from the site's H (upper triangle), then one stacked GPTQ solve of every weight
        that reads the site (outputs are views into stacked per-site buffers)."""
        d = site.d
        _lib.ctx_for(self.device.index)
        _lib.call("llmc_chol_inverse", self.c, C.c_void_p(h_ptr), C.c_int64(d), C.c_int64(d),
                  C.c_float(self.cfg.dampening_frac), 1, _lib.ptr(self.u), C.c_int64(d), 1)
        names = [w for w, _ in site.weights]
        ms = [m for _, m in site.weights]
        k = len(names)
        wp = (C.c_void_p * k)(*[weights[w].data_ptr() for w in names])
        mp = (C.c_int64 * k)(*ms)
        lp = (C.c_int64 * k)(*[weights[w].stride(0) for w in names])
        st = outputs[_stack_key(site)]
        wq = st.get("wq")
        if wq is None:
            wq = self.work[: sum(ms) * d].view(sum(ms), d)
        _lib.call("llmc_gptq_quantize_batch", self.c, C.c_int32(k), wp, mp, lp, _lib.dtype_code(weights[names[0]].dtype),
                  C.c_int64(d), _lib.ptr(self.u), C.c_int64(d), C.byref(self.qc), _lib.ptr(wq), C.c_int64(d),
                  _lib.ptr(st["codes"]), _lib.ptr(st["scales"]), _lib.ptr(st["zero_points"]))

    def alloc_outputs(self, layer_weights: dict):
        """Stacked per-site output buffers plus per-weight views into them."""
        outs = {}
        for s in self.sites:
            n = s.d
            M = sum(m for _, m in s.weights)
            stacked = {
                "codes": torch.empty(M, (n + 1) // 2 if self.cfg.num_bits <= 4 else n, dtype=torch.uint8,
                                     device=self.device),
                "scales": torch.empty(param_shape(self.cfg.strategy, M, n, self.cfg.group_size), dtype=torch.float32,
                                      device=self.device),
                "zero_points": torch.empty(param_shape(self.cfg.strategy, M, n, self.cfg.group_size), dtype=torch.int32,
                                           device=self.device),
            }
            if self.cfg.strategy == "tensor":
                stacked["scales"] = torch.empty(len(s.weights), dtype=torch.float32, device=self.device)
                stacked["zero_points"] = torch.empty(len(s.weights), dtype=torch.int32, device=self.device)
            if self.keep_wq:
                stacked["wq"] = torch.empty(M, n, dtype=torch.float32, device=self.device)
            outs[_stack_key(s)] = stacked
            r0 = 0
            for i, (wname, m) in enumerate(s.weights):
                view = {}
                for f, t in stacked.items():
                    view[f] = t[i:i + 1] if (self.cfg.strategy == "tensor" and f in ("scales", "zero_points")) \
                        else t[r0:r0 + m]
                outs[wname] = view
                r0 += m
        return outs

    def run_layer(self, acts: dict, weights: dict, outputs: dict):
        for s in self.sites:
            self.accumulate(s, acts[s.name])
            self.solve_site(s, self.hessian_ptr(s.name), weights, outputs)


def _stack_key(site: SiteSpec) -> str:
    return "__stacked__" + site.name


class _HView:
    def __init__(self, ptr, d):
        self.__cuda_array_interface__ = {"shape": (d, d), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}
