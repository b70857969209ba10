"""Layer-level GPTQ pipeline: the one-shot flow of GPTQModifier.OnStart/OnEnd
(src/LLMCompressorSharp.Core/Algorithms/Gptq/GPTQModifier.cs:59-137) for a stack of decoder
layers whose calibration activations are given per input site.

One Hessian per distinct input site (q/k/v share the attention input, gate/up the MLP
input); every weight that reads a site is quantised against that site's factor U.  The
result per weight is the packed int codes, scales and zero-points (plus, optionally, the
fp32 fake-quantised weight the reference returns).

Overlap (one GPU): ``run`` pipelines the layers over two library contexts on two streams.
While layer l is solved (Cholesky factor + GPTQ, mostly latency-bound kernels) on the solve
stream, layer l+1's Hessians accumulate on the Hessian stream; the Hessian context's
persistent kernel is capped to ``sm_count - reserve_sms`` SMs so the solve always finds SMs
free.  Hessians rotate through three handle sets, and events order every hand-off:
solve(l) waits for accumulate(l), and accumulate(l+3) waits for solve(l) before it resets
the buffer set they share.

Multi-GPU: calibration tokens are split across ranks; each rank accumulates its partial
H for every site, the partial Hessians are summed onto the layer's owner rank
(``torch.distributed.reduce`` over NCCL), and owners solve their layers (layers are dealt
round-robin).  In the row-sharded mode every Hessian is all-reduced instead and each rank
solves its own rows of every layer.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .errors import InvalidOperationError
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

    def __init__(self, sites, cfg, device: torch.device, chunk_rows: int = 65536, keep_wq: bool = False,
                 solver: str = "gptq"):
        """``cfg`` is a GPTQConfig (``solver="gptq"``) or a SparseGPTConfig (``solver="sparsegpt"``:
        every weight is pruned against the site's factor, outputs are the keep masks and the
        pruned fp32 weights)."""
        if solver not in ("gptq", "sparsegpt"):
            raise ValueError(f"unknown solver {solver}")
        self.solver = solver
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
        self.overlap = None

    def enable_overlap(self, reserve_sms: int = 28):
        """Switch ``run`` to the two-stream schedule described in the module docstring;
        ``reserve_sms`` SMs are kept free of the persistent Hessian kernel for the solve."""
        if self.overlap is None:
            self.overlap = _Overlap(self, reserve_sms)
        return self

    def close(self):
        for p in self.h.values():
            _lib.call("llmc_hessian_destroy", C.c_void_p(p))
        self.h = {}
        if self.overlap is not None:
            self.overlap.close()
            self.overlap = None

    def launch_count(self) -> int:
        """Kernels launched so far by the library contexts this pipeline uses."""
        n = _lib.launch_count(self.device.index)
        if self.overlap is not None:
            for c in [self.overlap.ch] + self.overlap.solve_contexts():
                v = C.c_int64()
                _lib.call("llmc_launch_count", C.c_void_p(c), C.byref(v))
                n += int(v.value)
        return n

    def check(self):
        """Waits for the job and raises the first deferred device error (overlap mode)."""
        if self.overlap is not None:
            self.overlap.check()

    def hessian_sms(self) -> int:
        """SMs the Hessian kernel runs on."""
        sm = torch.cuda.get_device_properties(self.device).multi_processor_count
        return self.overlap.hessian_sms if self.overlap is not None else sm

    def hessian_ptr(self, site: str) -> int:
        p = C.c_void_p()
        _lib.call("llmc_hessian_data", C.c_void_p(self.h[site]), C.byref(p))
        return p.value

    def accumulate(self, site: SiteSpec, x: torch.Tensor, out_h: torch.Tensor | None = None):
        """H_site = sum over chunks of X^T X (reset first).  Optionally copy H out."""
        _lib.ctx_for(self.device.index)
        self._accumulate_into(self.h[site.name], x)
        if out_h is not None:
            out_h.copy_(torch.as_tensor(_HView(self.hessian_ptr(site.name), site.d), device=self.device))

    def _accumulate_into(self, handle: int, x: torch.Tensor, ready=None):
        """Reset one Hessian handle and add X^T X over X in row chunks (on the handle's stream).
        ``ready`` marks rows of X that are still arriving on another stream: a CUDA event (all
        of X), or a list of (rows, event) in row order, the event completing once rows [0, rows)
        have arrived.  Each chunk [r0, r1) first waits for the first event with rows >= r1 (the
        last event when none covers r1), so accumulation follows the copy chunk by chunk."""
        stream = torch.cuda.current_stream(self.device)
        if isinstance(ready, torch.cuda.Event):
            stream.wait_event(ready)
            ready = None
        marks = list(ready or [])
        T = x.shape[0]
        waits = chunk_waits([r for r, _ in marks], T, self.chunk)
        h = C.c_void_p(handle)
        _lib.call("llmc_hessian_reset", h)
        for i, r0 in enumerate(range(0, T, self.chunk)):
            r1 = min(T, r0 + self.chunk)
            if waits[i] >= 0:
                stream.wait_event(marks[waits[i]][1])
            _lib.call("llmc_hessian_update", h, C.c_void_p(x.data_ptr() + r0 * x.stride(0) * x.element_size()),
                      _lib.dtype_code(x.dtype), C.c_int64(r1 - r0), C.c_int64(x.stride(0)))

    def _accumulate_many(self, handles: list, xs: list, ready=None):
        """``_accumulate_into`` for several Hessians at once (one per layer), chunk-interleaved:
        each row chunk is added to every handle before the next chunk's copy is waited for.  The
        tensors in ``xs`` have the same number of rows; ``ready`` marks the rows of the first one."""
        stream = torch.cuda.current_stream(self.device)
        if isinstance(ready, torch.cuda.Event):
            stream.wait_event(ready)
            ready = None
        marks = list(ready or [])
        T = xs[0].shape[0]
        if any(x.shape[0] != T for x in xs):
            raise ValueError("the layers' activations of one site need the same number of rows")
        waits = chunk_waits([r for r, _ in marks], T, self.chunk)
        hs = [C.c_void_p(h) for h in handles]
        for h in hs:
            _lib.call("llmc_hessian_reset", h)
        for i, r0 in enumerate(range(0, T, self.chunk)):
            r1 = min(T, r0 + self.chunk)
            if waits[i] >= 0:
                stream.wait_event(marks[waits[i]][1])
            for h, x in zip(hs, xs):
                _lib.call("llmc_hessian_update", h, C.c_void_p(x.data_ptr() + r0 * x.stride(0) * x.element_size()),
                          _lib.dtype_code(x.dtype), C.c_int64(r1 - r0), C.c_int64(x.stride(0)))

    def solve_site(self, site: SiteSpec, h_ptr: int, weights: dict, outputs: dict, ctx=None, rows=None, u=None,
                   work=None):
        """U from the site's H (upper triangle), then one stacked GPTQ solve of every weight
        that reads the site (outputs are views into stacked per-site buffers).  ``ctx`` is a
        library context bound to the stream to run on (default: torch's current stream).
        ``rows`` = (r0, r1) solves only those rows of the site's stack (rows are independent
        given U); the stacked outputs are written at the same rows.  Row ranges need a
        per-row strategy (channel or group).  ``u`` (d * d fp32) and ``work`` (the stack's rows
        * d fp32) are scratch buffers for this call; by default the pipeline's own, so solves
        that run at the same time on other streams pass their own."""
        from .distributed import stack_slices

        d = site.d
        if ctx is None:
            _lib.ctx_for(self.device.index)
            ctx = self.c
        names = [w for w, _ in site.weights]
        ms = [m for _, m in site.weights]
        M = sum(ms)
        r0, r1 = (0, M) if rows is None else (int(rows[0]), int(rows[1]))
        if not 0 <= r0 <= r1 <= M:
            raise ValueError(f"row range [{r0}, {r1}) outside the stack of {M} rows")
        if rows is not None and self.solver == "gptq" and self.cfg.strategy == "tensor":
            raise ValueError("row-sharded solves need a per-row strategy (channel or group)")
        u = self.u if u is None else u
        _lib.call("llmc_chol_inverse", ctx, C.c_void_p(h_ptr), C.c_int64(d), C.c_int64(d),
                  C.c_float(self.cfg.dampening_frac), 1, _lib.ptr(u), C.c_int64(d), 1)
        if r1 == r0:
            return
        parts = stack_slices(ms, r0, r1)  # [(weight index, first row, rows)]
        st = outputs[_stack_key(site)]
        wq = st.get("wq")
        if wq is None:
            wq = (self.work if work is None else work)[: (r1 - r0) * d].view(r1 - r0, d)
        else:
            wq = wq[r0:r1]
        if self.solver == "sparsegpt":
            q0 = 0
            for i, a, m in parts:
                w = weights[names[i]]
                _lib.call("llmc_sparsegpt_prune", ctx,
                          C.c_void_p(w.data_ptr() + a * w.stride(0) * w.element_size()), _lib.dtype_code(w.dtype),
                          C.c_int64(m), C.c_int64(d), C.c_int64(w.stride(0)), _lib.ptr(u), C.c_int64(d),
                          C.byref(self.qc), C.c_void_p(wq.data_ptr() + q0 * d * 4), C.c_int64(d),
                          C.c_void_p(st["mask"].data_ptr() + (r0 + q0) * d))
                q0 += m
            return
        k = len(parts)
        ws = [weights[names[i]] for i, _, _ in parts]
        wp = (C.c_void_p * k)(*[w.data_ptr() + a * w.stride(0) * w.element_size() for w, (_, a, _) in zip(ws, parts)])
        mp = (C.c_int64 * k)(*[m for _, _, m in parts])
        lp = (C.c_int64 * k)(*[w.stride(0) for w in ws])
        codes, scales, zps = st["codes"], st["scales"], st["zero_points"]
        _lib.call("llmc_gptq_quantize_batch", ctx, C.c_int32(k), wp, mp, lp, _lib.dtype_code(ws[0].dtype),
                  C.c_int64(d), _lib.ptr(u), C.c_int64(d), C.byref(self.qc), _lib.ptr(wq), C.c_int64(d),
                  C.c_void_p(codes.data_ptr() + r0 * codes.stride(0) * codes.element_size()),
                  C.c_void_p(scales.data_ptr() + r0 * (scales.stride(0) if scales.dim() > 1 else 1) * 4),
                  C.c_void_p(zps.data_ptr() + r0 * (zps.stride(0) if zps.dim() > 1 else 1) * 4))

    def alloc_outputs(self, layer_weights: dict):
        """Stacked per-site output buffers plus per-weight views into them."""
        outs = {}
        for s in self.sites:
            n = s.d
            M = sum(m for _, m in s.weights)
            if self.solver == "sparsegpt":
                stacked = {"mask": torch.empty(M, n, dtype=torch.uint8, device=self.device)}
                if self.keep_wq:
                    stacked["wq"] = torch.empty(M, n, dtype=torch.float32, device=self.device)
                outs[_stack_key(s)] = stacked
                r0 = 0
                for wname, m in s.weights:
                    outs[wname] = {f: t[r0:r0 + m] for f, t in stacked.items()}
                    r0 += m
                continue
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

    def site_order(self):
        """The order in which the overlapped schedule accumulates a layer's sites: widest first.
        A caller that copies the activations in (``acts_ready``) copies them in this order, so
        that the site with the most Hessian work per copied byte starts first and hides the rest
        of the copy."""
        return sorted(self.sites, key=lambda s: -s.d)

    def run_distributed(self, layers, acts, weights, outputs, world: int, rank: int, group=None, before_solve=None,
                        after_solve=None, hess_events=None, acts_ready=None, shard: str = "layers", sync: bool = True):
        """``run`` for one process per GPU (NCCL process group initialised by the caller):
        ``acts`` are this rank's token shard.  ``shard="layers"``: partial Hessians are reduced
        onto each layer's owner, which solves the whole layer; ``weights`` / ``outputs`` are
        needed for the layers this rank owns (``distributed.owned_layers``).  ``shard="rows"``:
        each Hessian is all-reduced, every rank factors it and solves its rows of every site's
        stack (``distributed.row_shard``, 64-row blocks); ``weights`` / ``outputs`` are needed for
        every layer and only this rank's rows of the stacked outputs are written.  Requires
        overlap enabled."""
        if self.overlap is None:
            raise InvalidOperationError("run_distributed needs enable_overlap() first")
        if shard not in ("layers", "rows"):
            raise ValueError(f"unknown shard mode {shard}")
        acts_for = acts if callable(acts) else (lambda _l: acts)
        return self.overlap.run_dist(list(layers), acts_for, weights, outputs, world, rank, group, before_solve,
                                     after_solve, hess_events, dict(acts_ready or {}), rows=shard == "rows", sync=sync)

    def run(self, layers, acts, weights, outputs, before_solve=None, after_solve=None, hess_events=None,
            acts_ready=None, sync: bool = True):
        """The whole job over ``layers``: per layer, every site's Hessian, factor and stacked
        GPTQ solve.  ``acts`` is {site: [T, d]} (shared by the layers) or a callable
        layer -> {site: tensor}; ``weights[l]`` / ``outputs[l]`` per layer.  ``before_solve(l)``
        and ``after_solve(l)`` run on the stream that solves layer l, just before / after it
        (e.g. host->device weight copies and device->host result copies).  With
        ``hess_events`` (a list), CUDA event pairs bracketing each site's accumulation are
        appended as (start, end, d, rows).  ``acts_ready`` ({site: CUDA event, or a list of
        (rows, event) per copied row range}) makes the first accumulation of each site wait for
        its activations, still being copied in on another stream (chunk by chunk with the list
        form).  Work is enqueued on the current stream (or, with overlap enabled,
        on the two pipeline streams joined back into it).  With overlap enabled the solves report a
        non-PD Hessian on the device; ``sync=True`` waits for the job at the end and raises such an
        error, ``sync=False`` returns at once and leaves the check to ``check()``."""
        acts_for = acts if callable(acts) else (lambda _l: acts)
        pending = dict(acts_ready or {})
        if self.overlap is not None:
            return self.overlap.run(list(layers), acts_for, weights, outputs, before_solve, after_solve, hess_events,
                                    pending, sync=sync)
        for l in layers:
            a = acts_for(l)
            for s in self.sites:
                ev = _events() if hess_events is not None else None
                if ev:
                    ev[0].record()
                _lib.ctx_for(self.device.index)
                self._accumulate_into(self.h[s.name], a[s.name], ready=pending.pop(s.name, None))
                if ev:
                    ev[1].record()
                    hess_events.append((ev[0], ev[1], s.d, a[s.name].shape[0]))
                if s is self.sites[0] and before_solve is not None:
                    before_solve(l)
                self.solve_site(s, self.hessian_ptr(s.name), weights[l], outputs[l])
            if after_solve is not None:
                after_solve(l)


def chunk_waits(mark_rows: list, T: int, chunk: int) -> list:
    """For each update chunk [r0, r1) of T rows, the index of the copy mark to wait for
    before it, or -1 when an earlier wait already covers it.  ``mark_rows`` are the row
    counts after which each mark's event completes, in order; a chunk waits for the first
    mark with rows >= r1, or the last mark when none reaches r1."""
    out, k, waited = [], 0, -1
    for r0 in range(0, T, chunk):
        r1 = min(T, r0 + chunk)
        if not mark_rows:
            out.append(-1)
            continue
        while k < len(mark_rows) - 1 and mark_rows[k] < r1:
            k += 1
        out.append(k if k != waited else -1)
        waited = k
    return out


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


class _Overlap:
    """Library contexts and streams for ``GptqPipeline.run``: one for the Hessians, one that
    orders each layer's solve (and the caller's copies around it), one per site for the site
    solves that run side by side; and rotating Hessian handle sets."""

    def __init__(self, pipe: GptqPipeline, reserve_sms: int):
        self.pipe = pipe
        dev = pipe.device
        sm = torch.cuda.get_device_properties(dev).multi_processor_count
        pr = torch.cuda.Stream.priority_range()
        hi, lo = min(pr), max(pr)  # a lower number is a higher priority
        # The Hessian stream is first in line for SMs at launch boundaries; the solve runs on
        # the reserved SMs (CTAs of a higher-priority stream do not overtake the pending CTAs
        # of a grid that is already being dispatched, so the split has to be static).
        self.sh = torch.cuda.Stream(dev, priority=hi)
        self.ss = torch.cuda.Stream(dev, priority=lo)
        self.ch = self._ctx(dev, self.sh)
        self.cs = self._ctx(dev, self.ss)
        limit = max(1, sm - int(reserve_sms))
        self.hessian_sms = limit
        _lib.call("llmc_set_sm_limit", C.c_void_p(self.ch), C.c_int32(limit))
        # The solve context shares the GPU: its tensor-core GEMMs launch one CTA per tile, which
        # start on the reserved SMs and on any SM a finishing Hessian launch frees.
        self.solve_sms = max(1, int(reserve_sms))
        _lib.call("llmc_set_sm_limit", C.c_void_p(self.cs), C.c_int32(self.solve_sms))
        # The factorisation decides a non-PD Hessian on the device, so enqueueing a solve never
        # waits for the GPU; a failure surfaces at the llmc_sync that ends the job.
        _lib.call("llmc_set_deferred_errors", C.c_void_p(self.cs), C.c_int32(1))
        # One stream, context and scratch set per site for ``run``: a layer's sites are
        # independent given their Hessians, so their solves (chains of mostly small, dependent
        # launches) run side by side on the reserved SMs instead of one after another.
        self.site_streams, self.site_ctx, self.site_u, self.site_work = [], [], [], []
        for site in pipe.sites:
            st = torch.cuda.Stream(dev, priority=lo)
            c = self._ctx(dev, st)
            _lib.call("llmc_set_sm_limit", C.c_void_p(c), C.c_int32(self.solve_sms))
            _lib.call("llmc_set_deferred_errors", C.c_void_p(c), C.c_int32(1))
            self.site_streams.append(st)
            self.site_ctx.append(c)
            self.site_u.append(torch.empty(site.d * site.d, dtype=torch.float32, device=dev))
            self.site_work.append(torch.empty(sum(m for _, m in site.weights) * site.d, dtype=torch.float32,
                                              device=dev))
        self.h = []
        self._ensure_sets(2)

    def _ensure_sets(self, n: int):
        """At least ``n`` Hessian handle sets (one handle per site each)."""
        while len(self.h) < n:
            hs = {}
            for s in self.pipe.sites:
                p = C.c_void_p()
                _lib.call("llmc_hessian_create", C.c_void_p(self.ch), C.c_int64(s.d), C.byref(p))
                hs[s.name] = p.value
            self.h.append(hs)

    @staticmethod
    def _ctx(dev, stream) -> int:
        out = C.c_void_p()
        _lib.call("llmc_init", C.c_int32(dev.index), C.byref(out))
        _lib.call("llmc_set_stream", out, C.c_void_p(stream.cuda_stream))
        return out.value

    def close(self):
        torch.cuda.synchronize(self.pipe.device)
        self.close_dist()
        for hs in self.h:
            for p in hs.values():
                _lib.call("llmc_hessian_destroy", C.c_void_p(p))
        self.h = []
        for c in [self.ch, self.cs] + self.site_ctx:
            _lib.call("llmc_destroy", C.c_void_p(c))
        self.ch = self.cs = None
        self.site_ctx, self.site_streams, self.site_u, self.site_work = [], [], [], []

    def solve_contexts(self) -> list:
        return [self.cs] + list(self.site_ctx)

    def _set_solve_limit(self, sms: int):
        for c in self.solve_contexts():
            _lib.call("llmc_set_sm_limit", C.c_void_p(c), C.c_int32(sms))

    def _data(self, b: int, site: str) -> int:
        p = C.c_void_p()
        _lib.call("llmc_hessian_data", C.c_void_p(self.h[b][site]), C.byref(p))
        return p.value

    # Layers whose Hessians accumulate site by site, chunk by chunk, while the calibration
    # activations are still arriving (``acts_ready``): every copied chunk then feeds this many
    # layers at once, so the first layers' work overlaps the copy instead of waiting for all of it.
    # On the Llama-3-8B job (52 GiB of activations, ≈ 1 s over PCIe) the end-to-end step measured
    # 9.66 / 9.58 / 9.46 / 9.41 s with 2 / 3 / 4 / 6 layers (one box, 1,300 MHz).
    PROLOGUE_LAYERS = 6

    def site_order(self):
        return self.pipe.site_order()

    def _hessian_whole_gpu(self, whole_gpu: bool):
        # Accumulations enqueued before the first solve have no solve beside them: they take
        # every SM (the limit is read when a launch is enqueued).
        _lib.call("llmc_set_sm_limit", C.c_void_p(self.ch), C.c_int32(0 if whole_gpu else self.hessian_sms))

    def _prologue(self, set_ids, sets, acts, acts_ready, hess_events, after_site):
        """Accumulates len(set_ids) layers at once on the current stream, site by site in
        ``site_order``, chunk-interleaved: each copied chunk of a site's activations is added to
        every layer's Hessian (``sets[set_ids[i]]``, from ``acts[i]``) before the next chunk is
        waited for.  ``after_site(site)`` runs on the stream after each site."""
        pipe = self.pipe
        for s in self.site_order():
            ev = _events() if hess_events is not None else None
            if ev:
                ev[0].record()
            pipe._accumulate_many([sets[b][s.name] for b in set_ids], [a[s.name] for a in acts],
                                  ready=acts_ready.pop(s.name, None))
            if ev:
                ev[1].record()
                hess_events.append((ev[0], ev[1], s.d, sum(a[s.name].shape[0] for a in acts)))
            after_site(s)

    def _enqueue_solve(self, l, h_ptrs: dict, weights, outputs, wait_ev, before_solve, after_solve, rows_for=None,
                       site_waits=None):
        """Enqueue the solve of layer l: the solve stream waits for ``wait_ev`` and runs the
        caller's ``before_solve``; each site then solves on its own stream and context (from the
        Hessian at ``h_ptrs[site]``, once ``site_waits[site]`` has completed when given;
        ``rows_for(site)`` picks a row range); the solve stream joins them and runs
        ``after_solve``.  Returns the event that marks the layer solved."""
        pipe = self.pipe
        with torch.cuda.stream(self.ss):
            self.ss.wait_event(wait_ev)
            if before_solve is not None:
                before_solve(l)
            start = torch.cuda.Event()
            start.record(self.ss)
        for j, s in enumerate(pipe.sites):
            st = self.site_streams[j]
            st.wait_event(start)
            if site_waits is not None:
                st.wait_event(site_waits[s.name])
            with torch.cuda.stream(st):
                pipe.solve_site(s, h_ptrs[s.name], weights[l], outputs[l], ctx=C.c_void_p(self.site_ctx[j]),
                                rows=rows_for(s) if rows_for is not None else None, u=self.site_u[j],
                                work=self.site_work[j])
                fin = torch.cuda.Event()
                fin.record(st)
            self.ss.wait_event(fin)
        with torch.cuda.stream(self.ss):
            if after_solve is not None:
                after_solve(l)
            done = torch.cuda.Event()
            done.record(self.ss)
        return done

    def run(self, layers, acts_for, weights, outputs, before_solve, after_solve, hess_events, acts_ready, sync=True):
        pipe = self.pipe
        cur = torch.cuda.current_stream(pipe.device)
        self.sh.wait_stream(cur)
        self.ss.wait_stream(cur)
        K = min(self.PROLOGUE_LAYERS, len(layers)) if acts_ready else 0
        if K < 2:
            K = 0
        # Three sets: the solve of layer l may run up to two layers' accumulation long before
        # layer l + 3 needs its set back, which absorbs solves that run long (the factorisation
        # of a layer whose Cholesky needs the damping fallback, launch jitter on the reserve).
        nsets = max(3, K + 1)
        self._ensure_sets(nsets)
        solved = [None] * nsets  # event: last solve that read buffer set b

        def solve(item):
            # item: (layer, set, event of the first site accumulated, events of every site)
            l, b, first_ev, site_evs = item
            solved[b] = self._enqueue_solve(l, {s.name: self._data(b, s.name) for s in pipe.sites}, weights, outputs,
                                            first_ev, before_solve, after_solve, site_waits=site_evs)

        def accumulated(s, evs):
            ev = torch.cuda.Event()
            ev.record(self.sh)
            evs[s.name] = ev

        hessian_limit = self._hessian_whole_gpu
        # Widest site first: its solve (the longest: the largest factorisation and GPTQ sweep)
        # starts while the narrower sites of the layer still accumulate, and each site's solve
        # waits only for its own Hessian.
        order = self.site_order()
        pending = None
        if K:
            # Prologue: layers 0..K-1 in sets 0..K-1, site-major, each arriving chunk added to
            # all K layers' Hessians before the next chunk is waited for.
            acts = [acts_for(l) for l in layers[:K]]
            hessian_limit(True)
            site_evs = {}
            with torch.cuda.stream(self.sh):
                self._prologue(list(range(K)), self.h, acts, acts_ready, hess_events,
                               lambda s: accumulated(s, site_evs))
            hessian_limit(False)
            first_ev = site_evs[order[0].name]
            for i in range(K - 1):
                solve((layers[i], i, first_ev, site_evs))
            pending = (layers[K - 1], K - 1, first_ev, site_evs)
        for i in range(K, len(layers)):
            l = layers[i]
            b = i % nsets
            a = acts_for(l)
            first = pending is None  # nothing solves beside this accumulation
            if first:
                hessian_limit(True)
            site_evs = {}
            with torch.cuda.stream(self.sh):
                if solved[b] is not None:
                    self.sh.wait_event(solved[b])
                for s in order:
                    ev = _events() if hess_events is not None else None
                    if ev:
                        ev[0].record(self.sh)
                    pipe._accumulate_into(self.h[b][s.name], a[s.name], ready=acts_ready.pop(s.name, None))
                    if ev:
                        ev[1].record(self.sh)
                        hess_events.append((ev[0], ev[1], s.d, a[s.name].shape[0]))
                    accumulated(s, site_evs)
            if first:
                hessian_limit(False)
            if pending is not None:
                solve(pending)
            pending = (l, b, site_evs[order[0].name], site_evs)
        if pending is not None:
            # The last layer's solve waits for the last accumulation, so nothing else runs beside
            # it: lift the solve context's SM limit (persistent grids over the whole GPU) for it.
            self._set_solve_limit(0)
            try:
                solve(pending)
            finally:
                self._set_solve_limit(self.solve_sms)
        cur.wait_stream(self.sh)
        cur.wait_stream(self.ss)
        if sync:
            self.check()

    def check(self):
        """Waits for the solve stream and raises the first deferred device error (a Hessian
        that was not positive definite, a bounded wait that gave up) of either context."""
        for c in self.solve_contexts() + [self.ch]:
            _lib.call("llmc_sync", C.c_void_p(c))

    # ---- one process per GPU ------------------------------------------------------------------
    DIST_SETS = 6  # Hessian handle sets in flight per rank
    # An owned layer's solve is enqueued once this many later layers are queued behind it.  The
    # solve stream waits for the layer's reduction on the device, so enqueueing never blocks the
    # host; one layer of lag keeps the next accumulation ahead of the solve in the launch order.
    DIST_LAG = 1

    def _dist_sets(self, n: int):
        if not getattr(self, "hd", None):
            self.hd = []
            self.sc = torch.cuda.Stream(self.pipe.device)
        while len(self.hd) < n:
            hs = {}
            for s in self.pipe.sites:
                p = C.c_void_p()
                _lib.call("llmc_hessian_create", C.c_void_p(self.ch), C.c_int64(s.d), C.byref(p))
                hs[s.name] = p.value
            self.hd.append(hs)
        return self.hd

    def close_dist(self):
        for hs in getattr(self, "hd", []):
            for p in hs.values():
                _lib.call("llmc_hessian_destroy", C.c_void_p(p))
        self.hd = []

    def run_dist(self, layers, acts_for, weights, outputs, world, rank, group, before_solve, after_solve,
                 hess_events, acts_ready, rows=False, sync=True):
        """Token-sharded job on `world` ranks: every rank accumulates its partial Hessians of
        every layer on the Hessian stream and reduces them onto the layer's owner with NCCL
        (issued from the Hessian stream, so the transfer of layer l overlaps the accumulation of
        layer l+1); owners solve on the solve stream once the reduction is done.  With ``rows``
        the reduction is an all-reduce and every rank solves its row shard of every layer."""
        import torch.distributed as dist

        from .distributed import layer_owner, row_shard

        pipe = self.pipe
        layers = list(layers)
        K = min(self.PROLOGUE_LAYERS, len(layers)) if acts_ready else 0
        if K < 2:
            K = 0
        # The prologue's K sets are reused only after their reductions (and owned solves): keep
        # half the steady-state sets free beyond them.
        sets = self._dist_sets(max(self.DIST_SETS, K + self.DIST_SETS // 2))
        cur = torch.cuda.current_stream(pipe.device)
        for st in (self.sh, self.ss, self.sc):
            st.wait_stream(cur)
        released = [None] * len(sets)  # event after which set b may be overwritten
        queue = []                      # owned layers waiting to be solved: (index, layer, set, reduce event)
        order = self.site_order()

        def solve(item):
            _, l, b, rd = item
            ptrs = {}
            for s in pipe.sites:
                p = C.c_void_p()
                _lib.call("llmc_hessian_data", C.c_void_p(sets[b][s.name]), C.byref(p))
                ptrs[s.name] = p.value
            rows_for = (lambda s: row_shard(sum(m for _, m in s.weights), world, rank)) if rows else None
            released[b] = self._enqueue_solve(l, ptrs, weights, outputs, rd, before_solve, after_solve, rows_for)

        def reduce(i, l, b):
            # Issued from the Hessian stream (NCCL waits for the accumulation); the copy stream
            # records when the reduction is done.  Every rank issues the same reductions in the
            # same order.
            with torch.cuda.stream(self.sh):
                works = []
                for s in order:
                    p = C.c_void_p()
                    _lib.call("llmc_hessian_data", C.c_void_p(sets[b][s.name]), C.byref(p))
                    h = torch.as_tensor(_HView(p.value, s.d), device=pipe.device)
                    if rows:
                        works.append(dist.all_reduce(h, op=dist.ReduceOp.SUM, group=group, async_op=True))
                    else:
                        works.append(dist.reduce(h, dst=layer_owner(l, world), op=dist.ReduceOp.SUM, group=group,
                                                 async_op=True))
            with torch.cuda.stream(self.sc):
                for w in works:
                    w.wait()
                rd = torch.cuda.Event()
                rd.record(self.sc)
            if rows or layer_owner(l, world) == rank:
                queue.append((i, l, b, rd))
            else:
                released[b] = rd
            while queue and queue[0][0] + self.DIST_LAG <= i:
                solve(queue.pop(0))

        if K:
            # Prologue, as on one GPU: layers 0..K-1 accumulate together while this rank's
            # activations are still arriving, on every SM; their reductions follow.
            self._hessian_whole_gpu(True)
            with torch.cuda.stream(self.sh):
                self._prologue(list(range(K)), sets, [acts_for(l) for l in layers[:K]], acts_ready, hess_events,
                               lambda s: None)
            self._hessian_whole_gpu(False)
            for i in range(K):
                reduce(i, layers[i], i)
        for i in range(K, len(layers)):
            l = layers[i]
            b = i % len(sets)
            a = acts_for(l)
            with torch.cuda.stream(self.sh):
                if released[b] is not None:
                    self.sh.wait_event(released[b])
                for s in order:
                    ev = _events() if hess_events is not None else None
                    if ev:
                        ev[0].record(self.sh)
                    pipe._accumulate_into(sets[b][s.name], a[s.name], ready=acts_ready.pop(s.name, None))
                    if ev:
                        ev[1].record(self.sh)
                        hess_events.append((ev[0], ev[1], s.d, a[s.name].shape[0]))
            reduce(i, l, b)
        if queue:
            # Solves enqueued after the last accumulation and reduction have nothing to share
            # the GPU with: persistent grids over every SM.
            self._set_solve_limit(0)
            try:
                while queue:
                    solve(queue.pop(0))
            finally:
                self._set_solve_limit(self.solve_sms)
        for st in (self.sh, self.ss, self.sc):
            cur.wait_stream(st)
        if sync:
            self.check()


def _stack_key(site: SiteSpec) -> str:
    return "__stacked__" + site.name


class _HView:
    def __init__(self, ptr, d):
        self.__cuda_array_interface__ = {"shape": (d, d), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}
