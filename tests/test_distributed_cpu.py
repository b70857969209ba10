"""Multi-GPU host logic on CPU: token shards, layer owners and the Hessian reduction, run as
world-size-2 gloo process groups (the GPU runs use the same functions over NCCL).

The partial Hessians here come from the oracle (this is a test of the partitioning and of
the exchange step, not of the CUDA kernels)."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llmcompressorsharp_b200.distributed import layer_owner, owned_layers, reduce_hessians, token_shard

SITES = [("attn_in", 48), ("down_in", 80)]
LAYERS = range(3)
TOKENS = 1001


def test_token_shards_partition_the_calibration_set():
    for tokens in (0, 1, 7, 100, 1001, 1_048_576):
        for world in (1, 2, 3, 8):
            parts = [token_shard(tokens, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == tokens
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        token_shard(10, 2, 2)


def test_layers_are_dealt_round_robin():
    world = 4
    owned = [owned_layers(range(32), world, r) for r in range(world)]
    assert sorted(sum(owned, [])) == list(range(32))
    assert all(len(o) == 8 for o in owned)
    assert all(layer_owner(l, world) == r for r in range(world) for l in owned[r])


def _acts():
    g = torch.Generator().manual_seed(7)
    return {name: torch.randn(TOKENS, d, generator=g) for name, d in SITES}


def _worker(rank, world, port, out_dir):
    from oracle import hessian as o_hess

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        acts = _acts()  # every rank sees the same calibration set and keeps its own shard
        r0, r1 = token_shard(TOKENS, world, rank)
        hbufs = {}
        for l in LAYERS:
            hbufs[l] = {}
            for name, d in SITES:
                acc = o_hess.HessianAccumulator(d)
                acc.update(acts[name][r0:r1] * (l + 1))
                hbufs[l][name] = acc.get_hessian()
        reduce_hessians(hbufs, [n for n, _ in SITES], LAYERS, world)
        mine = {l: hbufs[l] for l in owned_layers(LAYERS, world, rank)}
        torch.save(mine, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partial_hessians_reduce_onto_owners(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    from oracle import hessian as o_hess

    acts = _acts()
    got = {}
    for r in range(world):
        part = torch.load(tmp_path / f"rank{r}.pt")
        assert sorted(part) == owned_layers(LAYERS, world, r)
        got.update(part)
    assert sorted(got) == list(LAYERS)
    for l in LAYERS:
        for name, d in SITES:
            acc = o_hess.HessianAccumulator(d)
            acc.update(acts[name] * (l + 1))
            full = acc.get_hessian()
            assert torch.allclose(got[l][name], full, rtol=1e-5, atol=1e-3), (l, name)
