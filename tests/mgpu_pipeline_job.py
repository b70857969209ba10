"""Pipeline job for tests/test_multi_gpu.py (run under torchrun, one GPU per rank).

Every rank builds the same seeded calibration set and weights, keeps its token shard, and runs
``GptqPipeline.run_distributed`` in the mode given on the command line; it then solves the
whole job on its own GPU from the full token set and compares what it is responsible for
(its owned layers, or its rows of every layer) with that single-GPU result.  With a second
argument ``copied`` the shard starts in pinned host memory and is copied in chunk by chunk on
another stream while the job runs (``acts_ready``), over enough layers that the prologue runs
and its Hessian sets are reused.  Exit status 0 means every comparison held."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from llmcompressorsharp_b200 import GPTQConfig  # noqa: E402
from llmcompressorsharp_b200.distributed import owned_layers, row_shard, token_shard  # noqa: E402
from llmcompressorsharp_b200.pipeline import GptqPipeline, SiteSpec, _stack_key  # noqa: E402


def main():
    mode = sys.argv[1]
    copied = len(sys.argv) > 2 and sys.argv[2] == "copied"
    world, rank, local = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    sites = [SiteSpec("a", 256, [("w1", 320), ("w2", 64)]), SiteSpec("b", 512, [("w3", 256)])]
    layers, tokens = (10 if copied else 4), 12000
    g = torch.Generator().manual_seed(60)
    acts = {s.name: torch.randn(tokens, s.d, generator=g).to(torch.bfloat16).to(dev) for s in sites}
    weights = {l: {w: (torch.randn(m, s.d, generator=g) * 0.02).to(torch.bfloat16).to(dev)
                   for s in sites for w, m in s.weights} for l in range(layers)}
    cfg = GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=128)
    t0, t1 = token_shard(tokens, world, rank)
    shard = {k: v[t0:t1] for k, v in acts.items()}

    pipe = GptqPipeline(sites, cfg, dev, chunk_rows=4096).enable_overlap(24)
    mine = list(range(layers)) if mode == "rows" else owned_layers(range(layers), world, rank)
    outs = {l: pipe.alloc_outputs(weights[l]) for l in mine}
    ready = None
    if copied:
        host = {k: v.cpu().pin_memory() for k, v in shard.items()}
        shard = {k: torch.empty_like(v) for k, v in shard.items()}
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(torch.cuda.current_stream(dev))
        ready = {}
        with torch.cuda.stream(cs):
            for s in pipe.site_order():
                T, ready[s.name] = shard[s.name].shape[0], []
                for r0 in range(0, T, 1500):
                    r1 = min(T, r0 + 1500)
                    shard[s.name][r0:r1].copy_(host[s.name][r0:r1], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    ready[s.name].append((r1, ev))
    pipe.run_distributed(range(layers), shard, weights, outs, world, rank, shard=mode, acts_ready=ready)
    torch.cuda.synchronize()
    pipe.close()

    ref_pipe = GptqPipeline(sites, cfg, dev, chunk_rows=4096)
    ref = {l: ref_pipe.alloc_outputs(weights[l]) for l in mine}
    ref_pipe.run(mine, acts, weights, ref)
    torch.cuda.synchronize()
    ref_pipe.close()

    ok = True
    for l in mine:
        for s in sites:
            a, b = outs[l][_stack_key(s)], ref[l][_stack_key(s)]
            r0, r1 = row_shard(sum(m for _, m in s.weights), world, rank) if mode == "rows" else (0, None)
            same_params = torch.equal(a["scales"][r0:r1], b["scales"][r0:r1]) and torch.equal(
                a["zero_points"][r0:r1], b["zero_points"][r0:r1])
            agree = (a["codes"][r0:r1] == b["codes"][r0:r1]).float().mean().item()
            print(f"rank {rank} layer {l} site {s.name} rows [{r0}, {r1}) params equal {same_params} "
                  f"codes agree {agree:.6f}", flush=True)
            ok &= same_params and agree >= 0.999
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
