"""Multi-GPU host logic on CPU: token shards, layer owners, row shards and the Hessian
reduction, run as world-size-2 gloo process groups (the GPU runs use the same functions over
NCCL).

The partial Hessians here come from the oracle (this is a test of the partitioning and of
the exchange step, not of the CUDA kernels)."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llmcompressorsharp_b200.distributed import (layer_owner, owned_layers, reduce_hessians, row_shard, stack_slices,
                                                 token_shard)

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


def test_row_shards_partition_a_stack_in_whole_blocks():
    for rows in (0, 1, 63, 64, 65, 6144, 28672, 4096 + 1024 * 2):
        for world in (1, 2, 3, 8):
            parts = [row_shard(rows, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == rows
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            assert all(a % 64 == 0 or a == rows for a, _ in parts)
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 64
    with pytest.raises(ValueError):
        row_shard(10, 2, 0, align=0)


def test_stack_slices_cover_the_range_once():
    ms = [4096, 1024, 1024]  # q, k, v of a Llama-3-8B attention input
    for r0, r1 in ((0, 6144), (0, 64), (4000, 4200), (5120, 6144), (3072, 5248), (6144, 6144)):
        parts = stack_slices(ms, r0, r1)
        assert sum(m for _, _, m in parts) == r1 - r0
        offs = [0, 4096, 5120]
        rows = [offs[i] + a + k for i, a, m in parts for k in range(m)]
        assert rows == list(range(r0, r1))
        assert all(0 <= a and a + m <= ms[i] for i, a, m in parts)


ROW_SITE = (96, [("w1", 70), ("w2", 50)])  # d, stacked weights (rows 0-69 and 70-119)
ROW_TOKENS = 777


def _row_worker(rank, world, port, out_dir):
    from oracle import gptq as o_gptq
    from oracle import hessian as o_hess

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        d, ws = ROW_SITE
        g = torch.Generator().manual_seed(11)
        x = torch.randn(ROW_TOKENS, d, generator=g)
        weights = [torch.randn(m, d, generator=g) * 0.02 for _, m in ws]
        t0, t1 = token_shard(ROW_TOKENS, world, rank)
        acc = o_hess.HessianAccumulator(d)
        acc.update(x[t0:t1])
        h = acc.get_hessian()
        dist.all_reduce(h)  # every rank gets the full H
        u = o_hess.upper_factor(o_hess.hessian_inverse(h, 0.01))
        cfg = o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=32, block_size=32)
        r0, r1 = row_shard(sum(m for _, m in ws), world, rank, align=16)
        out = []
        for i, a, m in stack_slices([m for _, m in ws], r0, r1):
            wq, codes, scales, zps = o_gptq.gptq_quantize_u(weights[i][a:a + m], u, cfg)
            out.append((i, a, m, codes, torch.from_numpy(np.asarray(scales))))
        torch.save({"rows": (r0, r1), "parts": out}, os.path.join(out_dir, f"rows{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_row_sharded_solve_matches_whole_solve(tmp_path):
    """All-reduce of the partial Hessians, then each rank solves its rows of the stack: the
    ranks' rows together cover the stack once and equal the whole-weight solve."""
    from oracle import gptq as o_gptq
    from oracle import hessian as o_hess

    world = 2
    mp.spawn(_row_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    d, ws = ROW_SITE
    g = torch.Generator().manual_seed(11)
    x = torch.randn(ROW_TOKENS, d, generator=g)
    weights = [torch.randn(m, d, generator=g) * 0.02 for _, m in ws]
    acc = o_hess.HessianAccumulator(d)
    acc.update(x)
    u = o_hess.upper_factor(o_hess.hessian_inverse(acc.get_hessian(), 0.01))
    cfg = o_gptq.GPTQConfig(num_bits=4, symmetric=False, strategy="group", group_size=32, block_size=32)
    full = [o_gptq.gptq_quantize_u(w, u, cfg) for w in weights]
    covered = [torch.zeros(m, dtype=torch.int32) for _, m in ws]
    for r in range(world):
        res = torch.load(tmp_path / f"rows{r}.pt")
        for i, a, m, codes, scales in res["parts"]:
            covered[i][a:a + m] += 1
            assert (codes == full[i][1][a:a + m]).float().mean() >= 0.999
            assert np.array_equal(scales.numpy(), np.asarray(full[i][2])[a:a + m])
    assert all(bool((c == 1).all()) for c in covered)


def _dropout_worker(rank, world, port, out_dir):
    """Rank 1 leaves between steps (before the reduction); rank 0 must get an error from its
    next collective instead of waiting for ever."""
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        return  # leaves without joining the reduction (no collective in flight)
    hbufs = {0: {"attn_in": torch.ones(8, 8)}}
    t = time.monotonic()
    try:
        reduce_hessians(hbufs, ["attn_in"], [0], world)
        outcome = "completed"
    except Exception as e:  # noqa: BLE001 — any error from the collective is the expected outcome
        outcome = f"error {type(e).__name__}"
    with open(os.path.join(out_dir, "dropout.txt"), "w") as f:
        f.write(f"{outcome} {time.monotonic() - t:.1f}")


def test_a_rank_that_leaves_fails_the_next_reduction_within_the_timeout(tmp_path):
    """Failure detection on the host: with a short process-group timeout, the surviving rank's
    Hessian reduction ends with an error (gloo ranks on CPU; nothing runs on a GPU)."""
    world = 2
    mp.spawn(_dropout_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    outcome, secs = (tmp_path / "dropout.txt").read_text().rsplit(" ", 1)
    assert outcome.startswith("error"), outcome
    assert float(secs) < 60
