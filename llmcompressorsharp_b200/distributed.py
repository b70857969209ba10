"""Multi-GPU partitioning of the one-shot job: one process per GPU.

Calibration tokens are a bag (HessianAccumulator.Update sums X^T X over rows,
src/LLMCompressorSharp.TorchExtensions/Hessian/HessianAccumulator.cs:59-64), so every rank
accumulates partial Hessians over its own token shard and the partials sum exactly.  Layers
are independent given their Hessians (GPTQModifier.OnEndCore solves them one by one from the
unquantised model, src/LLMCompressorSharp.Core/Algorithms/Gptq/GPTQModifier.cs:119-136), so
each layer is solved by one owner rank, dealt round-robin.  The only exchange is the sum of
the partial Hessians onto each owner (``torch.distributed.reduce``; NCCL on GPUs, gloo in the
CPU tests).

Row sharding is the other partition: GPTQ and SparseGPT rows are independent given the factor U
(every step of GptqBlockQuantizer.Quantize except U itself is row-wise,
src/LLMCompressorSharp.Core/Algorithms/Gptq/GptqBlockQuantizer.cs:124-180).  Every rank then
receives the full H with one all-reduce, factors it, and solves its own rows of the site's
stacked weights (``row_shard`` / ``stack_slices``).
"""

from __future__ import annotations


def token_shard(tokens: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of the calibration set that `rank` accumulates (contiguous, sizes differ
    by at most one row)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(tokens, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def layer_owner(layer: int, world: int) -> int:
    """Rank that solves `layer` (round-robin)."""
    return layer % world


def owned_layers(layers, world: int, rank: int) -> list:
    return [l for l in layers if layer_owner(l, world) == rank]


def reduce_hessians(hbufs: dict, sites, layers, world: int, group=None) -> None:
    """Sum every rank's partial Hessian hbufs[layer][site] onto the layer's owner, in place.

    All ranks issue the same reductions in the same order (layers ascending, sites in
    order), asynchronously, then wait for all of them; non-owner buffers are left with
    partial sums that callers must not use."""
    import torch.distributed as dist

    reqs = []
    for l in layers:
        for s in sites:
            name = s.name if hasattr(s, "name") else s
            reqs.append(dist.reduce(hbufs[l][name], dst=layer_owner(l, world), op=dist.ReduceOp.SUM, group=group,
                                    async_op=True))
    for r in reqs:
        r.wait()


def row_shard(rows: int, world: int, rank: int, align: int = 64) -> tuple[int, int]:
    """Rows [r0, r1) of a stacked weight that `rank` solves: contiguous, in whole blocks of
    `align` rows (the solve kernel's CTA height) except at the end; ranks past the last block
    get an empty range."""
    if align < 1:
        raise ValueError("align must be positive")
    blocks = (rows + align - 1) // align
    b0, b1 = token_shard(blocks, world, rank)
    return min(rows, b0 * align), min(rows, b1 * align)


def stack_slices(ms, r0: int, r1: int) -> list:
    """The parts of stacked rows [r0, r1) that fall in each weight of a stack of weights with
    row counts `ms` (stacked in order): [(index, first row in the weight, row count)]."""
    out, off = [], 0
    for i, m in enumerate(ms):
        lo, hi = max(r0, off), min(r1, off + m)
        if hi > lo:
            out.append((i, lo - off, hi - lo))
        off += m
    return out
