#!/usr/bin/env python
"""GPTQ W4A16 (asym int4, group 128, damp 0.01, block 128) on a random-init Llama-3-8B-shaped
model with 512 x 2048 = 1,048,576 calibration tokens: wall-clock seconds per full job, with
the Hessian kernel's throughput and roofline.

One step = the whole one-shot job for all 32 decoder layers: per layer, the Hessian of each
of the 4 distinct input sites (attention input -> q/k/v, o input, MLP input -> gate/up, down
input) over all calibration tokens on tcgen05 tensor cores, the damped Cholesky factor U of
each, and the GPTQ column-block solve of all 7 weights producing packed int4 codes, scales
and zero-points.

Synthetic data (no network): weights bf16 ~N(0, 0.02) per layer; activations bf16 ~N(0, 1),
one seeded [tokens, d] set per input site, shared by all layers.  The activations (52 GiB)
are far larger than L2, so every timed step streams them from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun): calibration tokens are split across ranks; each rank accumulates partial
Hessians for every layer, layer by layer, and sums them onto the layer's owner over NCCL while
the next layer accumulates; owners (layers dealt round-robin) solve their layers on a second
stream: total work fixed ("strong").
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODELS = {
    "llama3-8b": {"name": "llama3-8b", "label": "Llama-3-8B", "hidden": 4096, "intermediate": 14336, "heads": 32,
                  "kv_heads": 8, "layers": 32},
    "llama3-70b": {"name": "llama3-70b", "label": "Llama-3-70B", "hidden": 8192, "intermediate": 28672, "heads": 64,
                   "kv_heads": 8, "layers": 80},
}
MODEL = dict(MODELS["llama3-8b"])
METRIC = "GPTQ W4A16 wall-clock s (Llama-3-8B shape)"
SPARSE_METRIC = "SparseGPT 2:4 wall-clock s (Llama-3-8B shape)"
UNIT = "s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["gptq", "sparsegpt", "solve", "smollm", "rtn", "smoothquant", "awq"],
                   default="gptq",
                   help="gptq: the GPTQ W4A16 job (default); sparsegpt: the same job pruning 2:4 with SparseGPT; "
                        "solve: the job's factor + GPTQ solve alone, Hessians given; smollm: GPTQ W4A16 of a "
                        "SmolLM2-135M-shaped fp32 model driven by its calibration forward (128 x 512 tokens); "
                        "rtn: RTN W4A16 g128 + min-max observer passes over the Llama-3-8B Linear weights; "
                        "smoothquant: SmoothQuant (alpha 0.5) + W8A8 weights on a Llama-2-7B shape; awq: AWQ "
                        "20-point grid search + scale apply on Llama-3-8B layers")
    p.add_argument("--model", choices=sorted(MODELS), default="llama3-8b",
                   help="layer shapes of the gptq / sparsegpt / solve workloads (the headline is llama3-8b)")
    p.add_argument("--layers", type=int, default=None, help="decoder layers (default: the model's)")
    p.add_argument("--tokens", type=int, default=512 * 2048)
    p.add_argument("--chunk", type=int, default=65536, help="calibration rows per Hessian update call")
    p.add_argument("--e2e-steps", type=int, default=2)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--reserve-sms", type=int, default=28,
                   help="1 GPU: SMs kept free of the Hessian kernel for the overlapped solve (0 = no overlap)")
    return p.parse_args()


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of this GPU during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
                power.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        loaded = [s for s, p in zip(sm, power) if p > 300] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------------------ helpers
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            j = json.load(f)
        return float(j["bf16_tflops"]), float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), float(j["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def sites_for(model):
    from llmcompressorsharp_b200.pipeline import llama_sites

    return llama_sites(model["hidden"], model["intermediate"], model["heads"], model["kv_heads"])


# ------------------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    from llmcompressorsharp_b200.distributed import owned_layers, reduce_hessians, token_shard
    from llmcompressorsharp_b200.gptq import GPTQConfig
    from llmcompressorsharp_b200.pipeline import GptqPipeline

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    sites = sites_for(MODEL)
    L = args.layers
    r0, r1 = token_shard(args.tokens, world, rank)
    T_local = r1 - r0
    sparse = args.workload == "sparsegpt"
    if sparse:
        from llmcompressorsharp_b200.sparsegpt import SparseGPTConfig

        cfg = SparseGPTConfig(sparsity=0.5, mask_structure="2:4", block_size=128, dampening_frac=0.01)
    else:
        cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128,
                         dampening_frac=0.01)
    mine = owned_layers(range(L), world, rank)

    # ---- synthetic inputs, resident in HBM
    g = torch.Generator(dev)
    acts = {}
    for i, s in enumerate(sites):
        g.manual_seed(1000 + 17 * rank + i)
        acts[s.name] = _randn_bf16(T_local, s.d, dev, g)
    weights = {}
    for l in mine:
        weights[l] = {}
        for si, s in enumerate(sites):
            for wi, (wname, m) in enumerate(s.weights):
                g.manual_seed(10_000 + 97 * l + 7 * si + wi)
                weights[l][wname] = _randn_bf16(m, s.d, dev, g, std=0.02)
    pipe = GptqPipeline(sites, cfg, dev, chunk_rows=args.chunk, solver="sparsegpt" if sparse else "gptq")
    if args.reserve_sms > 0:
        pipe.enable_overlap(args.reserve_sms)
    pipelined_dist = world > 1 and args.reserve_sms > 0
    outputs = {l: pipe.alloc_outputs(weights[l]) for l in mine}
    hbufs = None
    if world > 1 and not pipelined_dist:
        hbufs = {l: {s.name: torch.empty(s.d, s.d, dtype=torch.float32, device=dev) for s in sites} for l in range(L)}
    torch.cuda.synchronize()

    hess_events = []
    solve_events = []  # (start, end) of each overlapped layer solve, on the solve stream

    def solve_mark(l):
        e = torch.cuda.Event(enable_timing=True)
        e.record()  # the pipeline calls this with the solve stream current
        if solve_events and len(solve_events[-1]) == 1:
            solve_events[-1].append(e)
        else:
            solve_events.append([e])

    def step(record=False):
        """One full job; returns nothing (work is enqueued on the current stream)."""
        if world == 1:
            mark = solve_mark if record and args.reserve_sms > 0 else None
            pipe.run(range(L), acts, weights, outputs, before_solve=mark, after_solve=mark,
                     hess_events=hess_events if record else None, sync=False)
            return
        if pipelined_dist:
            pipe.run_distributed(range(L), acts, weights, outputs, world, rank,
                                 hess_events=hess_events if record else None, sync=False)
            return
        # phase 1: partial Hessians of every layer over this rank's tokens
        for l in range(L):
            for s in sites:
                if record:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                pipe.accumulate(s, acts[s.name], out_h=hbufs[l][s.name])
                if record:
                    e1.record()
                    hess_events.append((e0, e1, s.d, acts[s.name].shape[0]))
        # phase 2: sum partials onto each layer's owner (NCCL reduce, one group)
        reduce_hessians(hbufs, sites, range(L), world)
        # phase 3: owners solve
        for l in mine:
            for s in sites:
                pipe.solve_site(s, hbufs[l][s.name].data_ptr(), weights[l], outputs[l])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    launches0 = pipe.launch_count()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step(record=True)
    t1.record()
    barrier()
    clk = clocks.stop()
    pipe.check()  # deferred device errors of the timed steps (a non-PD Hessian, a wait that gave up)
    launches = pipe.launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    hess_ms = sum(a.elapsed_time(b) for a, b, _, _ in hess_events) / args.steps
    hess_launches = sum((rows + args.chunk - 1) // args.chunk for _, _, _, rows in hess_events)
    hess_flops_computed = sum(d * (d + 1) * rows for _, _, d, rows in hess_events)  # SYRK: d(d+1)T
    hess_flops_full = sum(2 * d * d * rows for _, _, d, rows in hess_events)
    tot_hess_ms = sum(a.elapsed_time(b) for a, b, _, _ in hess_events)
    # Overlapped solves only: the last layer of each step runs alone, on the whole GPU.
    solve_ms = sorted(ev[0].elapsed_time(ev[1]) for i, ev in enumerate(solve_events) if i % L != L - 1)
    if world > 1:
        t = torch.tensor([ms, hess_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, hess_ms = float(t[0]), float(t[1])

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, pipe, sites, acts, weights, outputs, mine, world, rank, local, hbufs)
    if world > 1:
        et = torch.tensor([e2e["value"] if e2e else 0.0], device=dev, dtype=torch.float64)
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
        if e2e:
            e2e["value"] = float(et[0])

    if rank == 0:
        burst, sustained, hbm, src = peaks()
        sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
        per_launch_flops = hess_flops_computed / max(1, hess_launches)
        per_launch_ms = tot_hess_ms / max(1, hess_launches)
        achieved = per_launch_flops / (per_launch_ms * 1e-3) / 1e12
        # The CPU sample is sized for the headline (Llama-3-8B) shapes.
        cpu = None if args.no_cpu_baseline or world > 1 or args.model != "llama3-8b" else cpu_baseline(args)
        line = {
            "metric": SPARSE_METRIC if sparse else METRIC, "value": round(ms / 1e3, 4), "unit": UNIT, "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": ("SparseGPT 2:4 (50 %) damp 0.01 block 128, " if sparse else
                                    "GPTQ W4A16 asym g128 damp 0.01 block 128, ") +
                                   f"{MODEL['label']} shape ({args.layers} layers x 7 Linear, hidden {MODEL['hidden']}, "
                                   f"intermediate {MODEL['intermediate']}, {MODEL['heads']}/{MODEL['kv_heads']} heads), "
                                   f"{args.tokens} calibration tokens ({args.tokens // 2048} x 2048), bf16",
                       "layers": args.layers, "tokens": args.tokens, "update_rows": args.chunk,
                       "parallelism": f"tokens split over {world} GPU(s), layers dealt round-robin",
                       "overlap": (f"solve of layer l on a second stream while later layers accumulate (and, "
                                   f"on N > 1, while their NCCL reductions run); Hessian kernel capped at "
                                   f"{args.reserve_sms} SMs fewer") if args.reserve_sms > 0 else "none",
                       "activations": "one seeded bf16 [tokens, d] set per input site, shared by all layers",
                       "l2": "inputs larger than L2 ({:.0f} GiB of activations streamed per step)".format(
                           sum(args.tokens * st.d * 2 for st in sites_for(MODEL)) / 2 ** 30)},
            "hessian_tflops": round(hess_flops_full / (tot_hess_ms * 1e-3) / 1e12 if tot_hess_ms else 0, 1),
            "hessian_tflops_note": "Hessian TFLOP/s with the full-GEMM count 2*d^2*T (the metric's definition); "
                                   "the kernel computes the symmetric half",
            "hessian_ms_per_step": round(hess_ms, 2),
            "solve_ms_per_layer_median": round(solve_ms[len(solve_ms) // 2], 2) if solve_ms else None,
            "solve_ms_per_layer_max": round(solve_ms[-1], 2) if solve_ms else None,
            "roofline": {"kernel": "syrk_tc2_kernel (Hessian H += X^T X, tcgen05 CTA pairs)", "bound": "tensor",
                         "achieved": round(achieved, 1), "peak": sustained, "unit": "TFLOP/s",
                         "frac": round(achieved / sustained, 3),
                         "peak_note": f"{src} sustained bf16 (kernel runs inside a ~{ms / 1e3:.0f} s step)",
                         "sms": pipe.hessian_sms(),
                         "frac_of_its_sms": round(achieved / (sustained * pipe.hessian_sms() / sm_count), 3),
                         "algorithmic": "d(d+1)T FLOP per launch (symmetric rank-k update of T tokens)",
                         "traffic": SYRK_TRAFFIC_PER_LAUNCH,
                         "traffic_note": "ncu DRAM read+write bytes per launch of this kernel version, averaged "
                                         "over the step's mix of d=4096 (1.47 GB) and d=14336 (20.4 GB) launches of "
                                         "65,536 tokens; their algorithmic bytes are 0.60 GB and 2.70 GB (X once + "
                                         "H upper triangle)"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    pipe.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


# DRAM bytes (read + write) per Hessian launch of this workload, from one ncu capture of the four
# site launches of a 65,536-token step at the default SM reserve (dram__bytes_read.sum +
# dram__bytes_write.sum, captured with `--layers 1 --tokens 65536 --steps 1 --warmup 1 --no-e2e
# --no-cpu-baseline`): d = 4096: 1.341 GB read + 0.131 GB written; d = 14336: 18.33 GB + 2.11 GB.
# A step has three d = 4096 launches for every d = 14336 launch, so the average launch moves
# (3 * 1.472 + 20.44) / 4 GB.  Re-capture whenever the Hessian kernel changes.
SYRK_TRAFFIC_PER_LAUNCH = (3 * 1.472e9 + 20.44e9) / 4


def _randn_bf16(m, n, dev, g, std=1.0):
    import torch

    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    rows = max(1, (1 << 28) // n)
    for r0 in range(0, m, rows):
        r1 = min(m, r0 + rows)
        out[r0:r1] = (torch.randn(r1 - r0, n, device=dev, generator=g) * std).to(torch.bfloat16)
    return out


# ------------------------------------------------------------------------------ end to end
def run_e2e(args, pipe, sites, acts, weights, outputs, mine, world, rank, local, hbufs):
    """Same job through the public API with HOST buffers: every step copies the weights of
    this rank's layers and the calibration activations from pinned host memory, runs the
    job, and copies codes/scales/zero-points back to pinned host memory."""
    import torch
    import torch.distributed as dist

    from llmcompressorsharp_b200.distributed import reduce_hessians

    dev = torch.device("cuda", local)
    h_acts = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in acts.items()}
    for k in acts:
        h_acts[k].copy_(acts[k])
    h_w = {l: {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in weights[l].items()} for l in mine}
    for l in mine:
        for k in weights[l]:
            h_w[l][k].copy_(weights[l][k])
    stacked = {l: {k: o for k, o in outputs[l].items() if k.startswith("__stacked__")} for l in mine}
    h_out = {l: {k: {f: torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for f, t in o.items()}
                 for k, o in stacked[l].items()} for l in mine}
    h2d = sum(t.numel() * t.element_size() for t in h_acts.values())
    h2d += sum(t.numel() * t.element_size() for l in mine for t in h_w[l].values())
    d2h = sum(t.numel() * t.element_size() for l in mine for o in h_out[l].values() for t in o.values())

    copy_stream = torch.cuda.Stream(dev)

    def copy_acts():
        """Host->device copy of each site's activations on a copy stream, in update-call
        chunks with one event per chunk, so accumulation follows the copy chunk by chunk."""
        copy_stream.wait_stream(torch.cuda.current_stream(dev))
        ready = {}
        with torch.cuda.stream(copy_stream):
            for k in [s.name for s in pipe.site_order() if s.name in acts]:
                T = acts[k].shape[0]
                ready[k] = []
                for r0 in range(0, T, args.chunk):
                    r1 = min(T, r0 + args.chunk)
                    acts[k][r0:r1].copy_(h_acts[k][r0:r1], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(copy_stream)
                    ready[k].append((r1, ev))
        return ready

    out_stream = torch.cuda.Stream(dev)

    def copy_weights():
        """Host->device copy of every owned layer's weights on the copy stream, after the
        activations, one event per layer: the solve of layer l waits only for its own."""
        evs = {}
        with torch.cuda.stream(copy_stream):
            for l in mine:
                for k in weights[l]:
                    weights[l][k].copy_(h_w[l][k], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                evs[l] = ev
        return evs

    def e2e_step():
        ready = copy_acts()
        if world == 1 or hbufs is None:  # one GPU, or the pipelined multi-GPU job
            wev = copy_weights()
            out_stream.wait_stream(torch.cuda.current_stream(dev))

            def load_weights(l):  # runs on the solve stream
                torch.cuda.current_stream(dev).wait_event(wev[l])

            def store_outputs(l):  # device->host on its own stream, beside the next solve
                done = torch.cuda.Event()
                done.record()
                out_stream.wait_event(done)
                with torch.cuda.stream(out_stream):
                    for k, o in stacked[l].items():
                        for f, t in o.items():
                            h_out[l][k][f].copy_(t, non_blocking=True)

            if world == 1:
                pipe.run(mine, acts, weights, outputs, before_solve=load_weights, after_solve=store_outputs,
                         acts_ready=ready)
            else:
                pipe.run_distributed(range(args.layers), acts, weights, outputs, world, rank,
                                     before_solve=load_weights, after_solve=store_outputs, acts_ready=ready)
            torch.cuda.current_stream(dev).wait_stream(out_stream)
            return
        for l in range(args.layers):
            for s in sites:
                if s.name in ready:
                    torch.cuda.current_stream(dev).wait_event(ready.pop(s.name)[-1][1])
                pipe.accumulate(s, acts[s.name], out_h=hbufs[l][s.name])
        reduce_hessians(hbufs, sites, range(args.layers), world)
        for l in mine:
            for k in weights[l]:
                weights[l][k].copy_(h_w[l][k], non_blocking=True)
            for s in sites:
                pipe.solve_site(s, hbufs[l][s.name].data_ptr(), weights[l], outputs[l])
            for k, o in stacked[l].items():
                for f, t in o.items():
                    h_out[l][k][f].copy_(t, non_blocking=True)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    e2e_step()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    t1.record()
    barrier()
    ms = t0.elapsed_time(t1) / args.e2e_steps
    if world > 1:  # bytes of the whole job: every rank's copies
        tb = torch.tensor([h2d, d2h], device=dev, dtype=torch.float64)
        dist.all_reduce(tb)
        h2d, d2h = float(tb[0]), float(tb[1])
    return {"value": round(ms / 1e3, 4), "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "steps": args.e2e_steps, "api": "llmcompressorsharp_b200.pipeline.GptqPipeline over the C ABI, host buffers"}


# ------------------------------------------------------------------------------ CPU side
def cpu_sample_seconds(threads: int, scale: float = 1.0):
    """Times the oracle (a PyTorch-CPU restatement of the reference's TorchSharp path) on a
    bounded sample of the job and extrapolates to the whole job as the reference runs it:
    GPTQModifier keeps one accumulator, one HessianInverseSolver.Compute and one
    GptqBlockQuantizer.Quantize per targeted weight (GPTQModifier.cs:73-94,119-136), so a
    Llama-3-8B layer costs 6 Hessians and factorisations at d = hidden, 1 at d = intermediate,
    and 7 solves.  Hessian time is linear in tokens (timed on a token sample at both widths);
    the factorisation is timed at d = hidden and scaled by d^3; each solve is fitted as
    a + b*m per width from two row counts (the column loop has a per-column cost that does not
    grow with m).  ``scale`` < 1 shrinks the samples (warm-up).  Returns (seconds, description)."""
    import torch

    from oracle import gptq as o_gptq, hessian as o_hess

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    hid, inter, L, T = MODEL["hidden"], MODEL["intermediate"], MODEL["layers"], 512 * 2048
    kv = MODEL["kv_heads"] * (hid // MODEL["heads"])

    def hess_per_token(d, tokens):
        x = torch.randn(tokens, d, generator=g).to(torch.bfloat16)
        acc = o_hess.HessianAccumulator(d)
        t = time.perf_counter()
        acc.update(x)
        return (time.perf_counter() - t) / tokens, acc.get_hessian()

    tok_h, tok_i = max(256, int(8192 * scale)), max(256, int(2048 * scale))
    ph_h, h = hess_per_token(hid, tok_h)
    ph_i, _ = hess_per_token(inter, tok_i)
    t = time.perf_counter()
    u = o_hess.upper_factor(o_hess.hessian_inverse(h, 0.01))
    t_f = time.perf_counter() - t  # HessianInverseSolver.Compute + U at d = hidden
    cfg = o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128)

    def solve_fit(n, upper, m0, m1):
        ts = []
        for m in (m0, m1):
            w = (torch.randn(m, n, generator=g) * 0.02).to(torch.bfloat16)
            t = time.perf_counter()
            o_gptq.gptq_quantize_u(w, upper, cfg)
            ts.append(time.perf_counter() - t)
        b = max(0.0, (ts[1] - ts[0]) / (m1 - m0))
        return max(0.0, ts[0] - b * m0), b, ts

    a_h, b_h, ts_h = solve_fit(hid, u, 64, 256)
    a_i, b_i, ts_i = solve_fit(inter, torch.eye(inter), 32, 128)  # timing does not depend on U's values
    solves = sum(a_h + b_h * m for m in (hid, kv, kv, hid, inter, inter)) + a_i + b_i * hid
    per_layer = T * (6 * ph_h + ph_i) + t_f * (6 + (inter / hid) ** 3) + solves
    total = per_layer * L
    desc = (f"oracle on {threads} host threads, as the reference runs it (one accumulator, factorisation and "
            f"solve per weight, 7 per layer): Hessians timed on {tok_h} tokens at d={hid} and {tok_i} at "
            f"d={inter}, Hessian inverse + U at d={hid} ({t_f:.2f} s, d^3 for d={inter}), GPTQ fitted a + b*m "
            f"from m=64/256 at n={hid} ({ts_h[0]:.2f}/{ts_h[1]:.2f} s) and m=32/128 at n={inter} "
            f"({ts_i[0]:.2f}/{ts_i[1]:.2f} s); x32 layers, 1,048,576 tokens. A lower bound on the reference, whose "
            "per-row P/Invoke loops this vectorised restatement does not pay")
    return total, desc


def cpu_baseline(args):
    threads = os.cpu_count() or 1
    total, desc = cpu_sample_seconds(threads)
    return {"value": round(total, 1), "unit": UNIT, "cores": threads, "kind": "port", "sample": desc}


def run_reference(args):
    """--impl reference: the reference's CPU algorithm (the oracle restatement; the C#/.NET
    reference cannot be built in this image) on all host threads, same metric and config."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    steps = []
    desc = ""
    threads = os.cpu_count() or 1
    if args.warmup > 0:
        cpu_sample_seconds(threads, 0.125)  # warm the CPU kernels once; a step is already seconds long
    for _ in range(args.steps):
        total, desc = cpu_sample_seconds(threads)
        steps.append(total)
    v = statistics.median(steps)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "GPTQ W4A16 asym g128, Llama-3-8B shape, 1,048,576 calibration tokens",
                       "layers": MODEL["layers"], "tokens": 512 * 2048},
            "cpu_baseline": {"value": round(v, 1), "unit": UNIT, "cores": threads, "kind": "port", "sample": desc},
            "e2e": {"value": round(v, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_solve(args):
    """--workload solve: the solve half of the GPTQ W4A16 job alone, on one GPU that it has to
    itself.  Every site's Hessian is accumulated once, before the timed region, from 2d seeded
    bf16 rows; a step then runs, for each of the layers and each site, the damped inverse factor
    U and the stacked GPTQ solve to packed codes, scales and zero-points (the same calls as the
    job's solve stream).  Algorithmic work per site: (2/3)d^3 for the factor (Cholesky and
    triangular inverse) + M d^2 for the solve's rank updates (M stacked rows), all in fp32."""
    import torch

    from llmcompressorsharp_b200.gptq import GPTQConfig
    from llmcompressorsharp_b200.pipeline import GptqPipeline

    world, rank, local = dist_env()
    if world > 1:
        raise SystemExit("--workload solve runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    sites = sites_for(MODEL)
    L = args.layers
    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128,
                     dampening_frac=0.01)
    pipe = GptqPipeline(sites, cfg, dev, chunk_rows=args.chunk)
    g = torch.Generator(dev)
    for i, st in enumerate(sites):
        g.manual_seed(3000 + i)
        x = _randn_bf16(2 * st.d, st.d, dev, g)
        pipe.accumulate(st, x)
        del x
    weights = {}
    for l in range(L):
        weights[l] = {}
        for si, st in enumerate(sites):
            for wi, (wname, m) in enumerate(st.weights):
                g.manual_seed(10_000 + 97 * l + 7 * si + wi)
                weights[l][wname] = _randn_bf16(m, st.d, dev, g, std=0.02)
    outputs = {l: pipe.alloc_outputs(weights[l]) for l in range(L)}
    hptr = {st.name: pipe.hessian_ptr(st.name) for st in sites}
    torch.cuda.synchronize()

    def step():
        for l in range(L):
            for st in sites:
                pipe.solve_site(st, hptr[st.name], weights[l], outputs[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches0 = pipe.launch_count()
    clocks = ClockSampler(0)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = pipe.launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    flops = L * sum(2 * st.d ** 3 / 3 + sum(m for _, m in st.weights) * st.d ** 2 for st in sites)
    achieved = flops / (ms * 1e-3) / 1e12
    _, sustained, _, src = peaks()
    # 3xTF32: three tf32 MMAs per fp32 product, tf32 at half the bf16 rate
    peak = sustained / 2 / 3
    line = {"metric": "GPTQ W4A16 solve wall-clock s, Hessians given (Llama-3-8B shape)", "value": round(ms / 1e3, 4),
            "unit": "s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"damped inverse factor + stacked GPTQ W4A16 asym g128 solve of {L} Llama-3-8B "
                                   f"layers x 4 sites (d 4096 x 3, 14336), Hessians from 2d seeded bf16 rows",
                       "layers": L, "l2": "inputs larger than L2 (each layer's weights 0.44 GB, U up to 0.82 GB)"},
            "solve_tflops": round(achieved, 1),
            "roofline": {"kernel": "whole solve (3xTF32 gemm_tc2 / gemm_tc GEMMs, Cholesky base blocks, GPTQ block "
                                   "kernel)", "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 3),
                         "peak_note": f"{src} sustained bf16 / 2 (tf32 rate) / 3 (3xTF32 MMAs per fp32 product)",
                         "algorithmic": "(2/3) d^3 + M d^2 fp32 FLOP per site and layer", "traffic": None},
            "gpu_launches": launches, "clocks": clk}
    print(json.dumps(line), flush=True)
    pipe.close()


SMOL = {"seqs": 128, "seq_len": 512, "batch": 16}


def _smol_layer_flops(shape) -> float:
    """fp32 algorithmic FLOP of one SmolLM2 layer's GPTQ job: Hessians d(d+1)T of the four
    distinct inputs, the damped factor (2/3)d^3 per input, the GPTQ rank updates m d^2 per weight."""
    T = SMOL["seqs"] * SMOL["seq_len"]
    h, i = shape.hidden, shape.intermediate
    kv = shape.kv_heads * shape.head_dim
    hess = (3 * h * (h + 1) + i * (i + 1)) * T
    factor = (3 * h ** 3 + i ** 3) * 2 / 3
    solve = (h + 2 * kv + h + 2 * i) * h * h + h * i * i
    return hess + factor + solve


def smol_cpu_sample(threads: int):
    """The oracle (and the torch CPU forward) on one decoder layer of the SmolLM2 job: the
    layer's forward and its four Hessians over 8,192 of the 65,536 tokens (scaled x8), the
    four factorisations and the seven GPTQ solves in full; x30 layers.  Returns (seconds for
    the whole job, description)."""
    import torch

    from llmcompressorsharp_b200.calibration import SHAPES, LlamaForCalibration
    from oracle import gptq as o_gptq, hessian as o_hess

    torch.set_num_threads(threads)
    shape = SHAPES["smollm2-135m"]
    one = type(shape)(**{**shape.__dict__, "layers": 1})
    model = LlamaForCalibration(one, dtype=torch.float32, seed=0)
    layer = model.model.layers[0]
    sample = 8192
    g = torch.Generator().manual_seed(2)
    x = torch.randn(sample // 512, 512, shape.hidden, generator=g)
    acts = {}
    def keep(name):
        def hook(mod, inp, out):
            acts.setdefault(name, inp[0])
        return hook

    hooks = [m.register_forward_hook(keep(n)) for n, m in layer.named_modules() if isinstance(m, torch.nn.Linear)]
    cos, sin = model.rope_tables(512, torch.float32)
    t = time.perf_counter()
    with torch.no_grad():
        layer(x, cos, sin)
    t_fwd = time.perf_counter() - t
    for hk in hooks:
        hk.remove()
    sites = {"self_attn.q_proj": ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"],
             "self_attn.o_proj": ["self_attn.o_proj"], "mlp.gate_proj": ["mlp.gate_proj", "mlp.up_proj"],
             "mlp.down_proj": ["mlp.down_proj"]}
    cfg = o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128)
    weights = dict(layer.named_modules())
    t_h = t_f = t_q = 0.0
    for site, names in sites.items():
        a = acts[site].reshape(-1, acts[site].shape[-1])
        acc = o_hess.HessianAccumulator(a.shape[1])
        t = time.perf_counter()
        acc.update(a)
        t_h += time.perf_counter() - t
        t = time.perf_counter()
        u = o_hess.upper_factor(o_hess.hessian_inverse(acc.get_hessian(), 0.01))
        t_f += time.perf_counter() - t
        for n in names:
            t = time.perf_counter()
            o_gptq.gptq_quantize_u(weights[n].weight.detach(), u, cfg)
            t_q += time.perf_counter() - t
    scale = SMOL["seqs"] * SMOL["seq_len"] / sample
    per_layer = (t_fwd + t_h) * scale + t_f + t_q
    desc = (f"oracle + torch CPU forward on {threads} host threads, one SmolLM2 layer: forward {t_fwd:.2f} s and "
            f"Hessians {t_h:.2f} s over 8,192 tokens (x8), 4 factorisations {t_f:.2f} s, 7 GPTQ solves {t_q:.2f} s; "
            "x30 layers")
    return per_layer * shape.layers, desc


def run_smollm(args):
    """--workload smollm: GPTQ W4A16 (asym int4 g128, damp 0.01, block 128) of a random-init
    SmolLM2-135M-shaped LLaMA (30 layers, hidden 576, intermediate 1536, 9 / 3 heads, vocab
    49152) with fp32 weights ~N(0, 0.02), calibrated on 128 x 512 uniform-random token ids run
    through the model: the reference's own CPU-runnable configuration.  A step is one
    CompressionSession with GPTQModifier (shared inputs deduplicated) driven by the calibration
    forward (``calibration.drive``): every Hessian update is the fp32 3xTF32 path, then the
    factor and the GPTQ solve of all 210 weights.  The forward is torch (cuBLAS); it is also
    timed alone."""
    import torch

    from llmcompressorsharp_b200 import _lib
    from llmcompressorsharp_b200.calibration import SHAPES, LlamaForCalibration, calibration_batches, drive
    from llmcompressorsharp_b200.gptq import GPTQConfig, GPTQModifier
    from llmcompressorsharp_b200.session import CompressionSession, CompressionState, SessionStatus

    world, _, _ = dist_env()
    if world > 1:
        raise SystemExit("--workload smollm runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    shape = SHAPES["smollm2-135m"]
    model = LlamaForCalibration(shape, dtype=torch.float32, device=dev, seed=0)
    batches = list(calibration_batches(shape.vocab, SMOL["seqs"], SMOL["seq_len"], SMOL["batch"], seed=1, device=dev))
    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128, block_size=128,
                     dampening_frac=0.01)

    def step():
        state = CompressionState(model.linear_weights())
        state.named_modules = model.linear_modules()
        session = CompressionSession([GPTQModifier(cfg, share_inputs=True)])
        if session.run(state, drive(model, batches)) != SessionStatus.COMPLETED:
            raise RuntimeError(f"GPTQ session failed: {session.failure!r}")
        return state

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for b in batches:
        model(b)
    f1.record()
    torch.cuda.synchronize()
    fwd_ms = f0.elapsed_time(f1)
    launches0 = _lib.launch_count(0)
    clocks = ClockSampler(0)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        state = step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = _lib.launch_count(0) - launches0
    ms = t0.elapsed_time(t1) / args.steps
    codes = sum(1 for e in state.compressed.values() if e.get("codes") is not None)
    flops = _smol_layer_flops(shape) * shape.layers
    _, sustained, _, src = peaks()
    peak = sustained / 2 / 3
    achieved = flops / ((ms - fwd_ms) * 1e-3) / 1e12
    cpu = None
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        total, desc = smol_cpu_sample(threads)
        cpu = {"value": round(total, 1), "unit": "s", "cores": threads, "kind": "port", "sample": desc}
    line = {"metric": "GPTQ W4A16 wall-clock s (SmolLM2-135M shape, fp32, calibration forward included)",
            "value": round(ms / 1e3, 4), "unit": "s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 2), "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "GPTQ W4A16 asym g128 damp 0.01 block 128 of a random-init SmolLM2-135M-shaped "
                                   "LLaMA (30 layers, hidden 576, intermediate 1536, 9/3 heads), fp32 weights "
                                   "N(0, 0.02), 128 x 512 uniform-random token ids through the model in batches of 16",
                       "weights_quantised": codes, "l2": "weights (0.5 GB fp32) and activations larger than L2"},
            "forward_ms": round(fwd_ms, 2),
            "roofline": {"kernel": "whole step less the forward: fp32 Hessians (3xTF32 gemm_tc2 with token splits), "
                                   "factorisations, GPTQ solves", "bound": "tensor", "achieved": round(achieved, 1),
                         "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 3),
                         "peak_note": f"{src} sustained bf16 / 2 (tf32 rate) / 3 (3xTF32 MMAs per fp32 product)",
                         "algorithmic": "Hessians d(d+1)T + factors (2/3)d^3 + GPTQ m d^2, fp32", "traffic": None},
            "cpu_baseline": cpu, "e2e": None, "gpu_launches": launches, "clocks": clk}
    print(json.dumps(line), flush=True)


def run_rtn(args):
    """RTN W4A16 (asym int4, group 128) quantise+pack and a group-128 min-max observer pass
    over every Linear weight of a Llama-3-8B-shaped model (224 bf16 weights, 7.0 G params),
    each pass captured once in a CUDA graph and replayed.  Throughput is the algorithmic
    bytes of a pass (read W; write packed codes, scales and zero-points) over its device
    time; N > 1 deals the layers round-robin."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    from llmcompressorsharp_b200 import _lib
    from llmcompressorsharp_b200.distributed import owned_layers
    from llmcompressorsharp_b200.rtn import RtnConfig

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    sites = sites_for(MODEL)
    mine = owned_layers(range(args.layers), world, rank)
    g = torch.Generator(dev)
    ws = []
    for l in mine:
        for si, s in enumerate(sites):
            for wi, (_, m) in enumerate(s.weights):
                g.manual_seed(10_000 + 97 * l + 7 * si + wi)
                w = _randn_bf16(m, s.d, dev, g, std=0.02)
                hot = torch.rand(m, s.d, device=dev, generator=g) < 0.001  # 0.1 % outliers x20
                w[hot] *= 20
                ws.append(w)
    cfg = RtnConfig(num_bits=4, symmetric=False, strategy="group", group_size=128).to_c()
    outs = []
    for w in ws:
        m, n = w.shape
        outs.append((torch.empty(m, n // 2, dtype=torch.uint8, device=dev),
                     torch.empty(m, n // 128, dtype=torch.float32, device=dev),
                     torch.empty(m, n // 128, dtype=torch.int32, device=dev)))
    params = sum(w.numel() for w in ws)
    rtn_bytes = params * 2 + params // 2 + (params // 128) * 8
    obs_bytes = params * 2 + (params // 128) * 8

    def rtn_pass():
        c = C.c_void_p(_lib.ctx_for(local))
        for w, (codes, sc, zp) in zip(ws, outs):
            m, n = w.shape
            _lib.call("llmc_rtn_quantize", c, _lib.ptr(w), _lib.DTYPE_BF16, C.c_int64(m), C.c_int64(n), C.c_int64(n),
                      C.byref(cfg), _lib.ptr(codes), _lib.ptr(sc), _lib.ptr(zp), C.c_void_p(0))

    def observer_pass():
        c = C.c_void_p(_lib.ctx_for(local))
        for w, (_, sc, zp) in zip(ws, outs):
            m, n = w.shape  # min -> scales buffer, max -> zero-point buffer (same size, 4-byte elements)
            _lib.call("llmc_observer_minmax", c, _lib.ptr(w), _lib.DTYPE_BF16, C.c_int64(m), C.c_int64(n), C.c_int64(n),
                      _lib.STRATEGY["group"], C.c_int64(128), _lib.ptr(sc), _lib.ptr(zp), 0)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    launches0 = _lib.launch_count(local)
    graphs = {}
    for name, fn in (("rtn", rtn_pass), ("observer", observer_pass)):
        fn()  # first call outside capture (one-time set-up)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        graphs[name] = gr
    kernels_per_pass = (_lib.launch_count(local) - launches0) // 4

    def timed(gr):
        for _ in range(args.warmup):
            gr.replay()
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            gr.replay()
        t1.record()
        barrier()
        ms = t0.elapsed_time(t1) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        return ms

    clocks = ClockSampler(local)
    clocks.start()
    ms_rtn = timed(graphs["rtn"])
    ms_obs = timed(graphs["observer"])
    clk = clocks.stop()
    tot = torch.tensor([rtn_bytes, obs_bytes, params], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tot)
    rtn_all, obs_all, params_all = (float(v) for v in tot)

    # e2e through the public API with host buffers: weights in from pinned memory, codes,
    # scales and zero-points back out, every step.
    h_w = [torch.empty(w.shape, dtype=w.dtype, pin_memory=True) for w in ws]
    for hw, w in zip(h_w, ws):
        hw.copy_(w)
    h_o = [tuple(torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in o) for o in outs]

    def e2e_step():
        for hw, w in zip(h_w, ws):
            w.copy_(hw, non_blocking=True)
        rtn_pass()
        for ho, o in zip(h_o, outs):
            for a, b in zip(ho, o):
                a.copy_(b, non_blocking=True)

    e2e_step()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(max(1, args.e2e_steps)):
        e2e_step()
    t1.record()
    barrier()
    e2e_ms = t0.elapsed_time(t1) / max(1, args.e2e_steps)
    h2d = sum(t.numel() * t.element_size() for t in h_w)
    d2h = sum(t.numel() * t.element_size() for o in h_o for t in o)
    te = torch.tensor([e2e_ms, h2d, d2h], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(te[1:])
    e2e_ms, h2d, d2h = float(te[0]), float(te[1]), float(te[2])

    if rank == 0:
        _, _, hbm, src = peaks()
        per_gpu = rtn_bytes / (ms_rtn * 1e-3) / 1e9
        line = {
            "metric": "RTN W4A16 g128 quantise+pack throughput (Llama-3-8B Linear weights)",
            "value": round(rtn_all / (ms_rtn * 1e-3) / 1e9, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_rtn, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"RTN asym int4 group 128 over {len(ws)} bf16 Linear weights of {len(mine)} "
                                   f"Llama-3-8B layers on rank 0 ({int(params_all)} params in all)",
                       "bytes_per_param": "2 read + 0.5 codes + 8/128 scale and zero-point",
                       "l2": "inputs larger than L2 (14 GB of weights per pass)",
                       "launch": "each pass is one CUDA graph replay"},
            "observer_gbs": round(obs_all / (ms_obs * 1e-3) / 1e9, 1),
            "observer_ms_per_step": round(ms_obs, 3),
            "roofline": {"kernel": "rtn_kernel<bf16, 8> (fused group observer + fake-quant + int4 pack)",
                         "bound": "hbm", "achieved": round(per_gpu, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(per_gpu / hbm, 3), "peak_note": f"{src} HBM copy bandwidth",
                         "traffic": None},
            "e2e": {"value": round(rtn_all / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "api": "llmc_rtn_quantize over the C ABI, host buffers"},
            "gpu_launches": kernels_per_pass * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_smooth_awq(args):
    """--workload smoothquant: per layer of a Llama-2-7B shape (hidden 4096, intermediate 11008,
    32 layers, 256 x 2048 = 524,288 calibration tokens), the activation absmax of the attention
    and MLP inputs, SmoothQuant (alpha 0.5) of input_layernorm -> q/k/v and post_attention_layernorm
    -> gate/up, W8A8's int8 per-channel weight quantisation of all seven weights, and W8A8's int8
    per-token quantisation of the two activation inputs (codes and per-token scales).
    --workload awq: per layer of a Llama-3-8B shape (128 x 2048 = 262,144 tokens), the activation
    absmax of the same two inputs, the AWQ 20-point grid search (RTN asym int4 g128) and the
    scale apply for q/k/v and gate/up.  Both are HBM-bound: throughput = algorithmic bytes /
    device time; one GPU."""
    import ctypes as C

    import torch

    from llmcompressorsharp_b200 import _lib
    from llmcompressorsharp_b200.rtn import RtnConfig

    world, rank, local = dist_env()
    if world > 1:
        raise SystemExit("--workload smoothquant / awq run on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    awq = args.workload == "awq"
    hid = 4096
    inter = 14336 if awq else 11008
    kv = 1024 if awq else 4096
    T = 128 * 2048 if awq else 256 * 2048
    L = args.layers
    g = torch.Generator(dev).manual_seed(5)
    acts = []
    for _ in range(2):
        x = _randn_bf16(T, hid, dev, g)
        hot = torch.randperm(hid, device=dev, generator=g)[: hid // 100]  # 1 % heavy-tailed channels x50
        x[:, hot] = (x[:, hot].float() * 50 * torch.rand(T, hot.numel(), device=dev, generator=g).pow(-0.5)).to(x.dtype)
        acts.append(x)
    shapes = {"qkv": (hid + 2 * kv, hid), "o": (hid, hid), "gu": (2 * inter, hid), "down": (hid, inter)}
    layers = []
    for l in range(L):
        g.manual_seed(20_000 + l)
        w = {k: _randn_bf16(m, n, dev, g, std=0.02) for k, (m, n) in shapes.items()}
        w["ln1"] = (1 + 0.1 * torch.randn(hid, device=dev, generator=g)).to(torch.bfloat16)
        w["ln2"] = (1 + 0.1 * torch.randn(hid, device=dev, generator=g)).to(torch.bfloat16)
        layers.append(w)
    amax = [torch.empty(hid, device=dev) for _ in range(2)]
    s_out = torch.empty(hid, device=dev)
    n_grid = 20
    mse = torch.empty(n_grid, dtype=torch.float64, device=dev)
    q8 = RtnConfig(num_bits=8, symmetric=True, strategy="channel").to_c()
    q4 = RtnConfig(num_bits=4, symmetric=False, strategy="group", group_size=128).to_c()
    codes = {k: torch.empty(m, n, dtype=torch.uint8, device=dev) for k, (m, n) in shapes.items()}
    scales = {k: torch.empty(m, 1, dtype=torch.float32, device=dev) for k, (m, n) in shapes.items()}
    zps = {k: torch.empty(m, 1, dtype=torch.int32, device=dev) for k, (m, n) in shapes.items()}
    act_codes = act_scales = None
    if not awq:
        act_codes = torch.empty(T, hid, dtype=torch.int8, device=dev)
        act_scales = torch.empty(T, dtype=torch.float32, device=dev)

    def step():
        c = C.c_void_p(_lib.ctx_for(0))
        for w in layers:
            for x, am in zip(acts, amax):
                _lib.call("llmc_act_absmax", c, _lib.ptr(x), _lib.DTYPE_BF16, C.c_int64(T), C.c_int64(hid),
                          C.c_int64(hid), _lib.ptr(am), 0)
            for am, ln, key in ((amax[0], "ln1", "qkv"), (amax[1], "ln2", "gu")):
                m = shapes[key][0]
                if awq:
                    _lib.call("llmc_awq_search", c, _lib.ptr(w[key]), _lib.DTYPE_BF16, C.c_int64(m), C.c_int64(hid),
                              C.c_int64(hid), _lib.ptr(am), C.c_int32(n_grid), C.byref(q4), _lib.ptr(s_out),
                              _lib.ptr(mse), C.c_void_p(0))  # best_s is applied on the device: no read-back
                    _lib.call("llmc_scale_apply", c, _lib.ptr(s_out), _lib.ptr(w[ln]), _lib.DTYPE_BF16,
                              _lib.ptr(w[key]), _lib.DTYPE_BF16, C.c_int64(m), C.c_int64(hid))
                else:
                    _lib.call("llmc_smooth_apply", c, _lib.ptr(am), _lib.ptr(w[ln]), _lib.DTYPE_BF16,
                              _lib.ptr(w[key]), _lib.DTYPE_BF16, C.c_int64(m), C.c_int64(hid), C.c_float(0.5),
                              _lib.ptr(s_out))
            if not awq:
                for key, (m, n) in shapes.items():
                    _lib.call("llmc_rtn_quantize", c, _lib.ptr(w[key]), _lib.DTYPE_BF16, C.c_int64(m), C.c_int64(n),
                              C.c_int64(n), C.byref(q8), _lib.ptr(codes[key]), _lib.ptr(scales[key]),
                              _lib.ptr(zps[key]), C.c_void_p(0))
                for x in acts:  # the A side of W8A8: int8 per token, symmetric
                    _lib.call("llmc_act_quant_per_token", c, _lib.ptr(x), _lib.DTYPE_BF16, C.c_int64(T), C.c_int64(hid),
                              C.c_int64(hid), C.c_int32(8), C.c_int32(1), _lib.ptr(act_codes), C.c_int64(hid),
                              _lib.ptr(act_scales), C.c_void_p(0), C.c_void_p(0), C.c_int64(hid))

    # algorithmic bytes of one step
    absmax_b = 2 * T * hid * 2
    bal = (shapes["qkv"][0] + shapes["gu"][0]) * hid * 2
    if awq:
        per_layer = absmax_b + (n_grid + 1) * bal + 2 * bal + 4 * hid * 2
    else:
        params = sum(m * n for m, n in shapes.values())
        per_layer = absmax_b + 3 * bal + 4 * hid * 2 + params * 3 + sum(m for m, _ in shapes.values()) * 8
        per_layer += 2 * (T * hid * 2 + T * hid + T * 4)  # per-token: read x, write codes and scales
    step_bytes = per_layer * L
    launches0 = _lib.launch_count(0)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    warm_launches = (_lib.launch_count(0) - launches0) // max(1, args.warmup)
    clocks = ClockSampler(0)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    _, _, hbm, src = peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    name = ("AWQ grid search (20 points, int4 g128) + scale apply throughput (Llama-3-8B shape)" if awq else
            "SmoothQuant (alpha 0.5) + W8A8 (int8 per-channel weights, int8 per-token activations) throughput "
            "(Llama-2-7B shape)")
    line = {"metric": name, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{L} layers, {T} calibration tokens, hidden {hid}, intermediate {inter}",
                       "bytes_per_step": int(step_bytes),
                       "activations": "two [tokens, 4096] bf16 inputs, 1 % of channels heavy-tailed x50",
                       "l2": "inputs larger than L2"},
            "roofline": {"kernel": "awq_err_group_kernel" if awq else "col_absmax_kernel", "bound": "hbm",
                         "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 3),
                         "peak_note": f"{src} HBM copy bandwidth; whole-step bytes over step time", "traffic": None},
            "gpu_launches": warm_launches * args.steps, "clocks": clk}
    print(json.dumps(line), flush=True)


def main():
    global METRIC, SPARSE_METRIC
    args = parse()
    MODEL.clear()
    MODEL.update(MODELS[args.model])
    if args.layers is None:
        args.layers = MODEL["layers"]
    METRIC = f"GPTQ W4A16 wall-clock s ({MODEL['label']} shape)"
    SPARSE_METRIC = f"SparseGPT 2:4 wall-clock s ({MODEL['label']} shape)"
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "rtn":
        run_rtn(args)
        return
    if args.workload in ("smoothquant", "awq"):
        run_smooth_awq(args)
        return
    if args.workload == "solve":
        run_solve(args)
        return
    if args.workload == "smollm":
        run_smollm(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()
