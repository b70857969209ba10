"""Two-rank Hessian reduction through the C ABI for tests/test_multi_gpu.py (run under
torchrun, one GPU per rank): rank 0 makes an NCCL unique id with llmc_nccl_unique_id, the
ranks share it over a gloo group, open a communicator with llmc_nccl_comm_init, accumulate
their token shards and call llmc_hessian_allreduce (then llmc_hessian_reduce onto rank 1).
Every rank checks the summed H and sample count against a one-GPU accumulation of all tokens."""

import ctypes as C
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from llmcompressorsharp_b200 import HessianAccumulator, _lib  # noqa: E402
from llmcompressorsharp_b200.distributed import token_shard  # noqa: E402


def main():
    world, rank, local = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()
    ctx = C.c_void_p(_lib.ctx_for(local))
    uid = (C.c_uint8 * _lib.NCCL_UNIQUE_ID_BYTES)()
    if rank == 0:
        _lib.call("llmc_nccl_unique_id", C.cast(uid, C.c_void_p), C.c_int64(len(uid)))
    box = [bytes(uid)]
    dist.broadcast_object_list(box, src=0)
    uid = (C.c_uint8 * len(box[0])).from_buffer_copy(box[0])
    comm = C.c_void_p()
    _lib.call("llmc_nccl_comm_init", ctx, C.c_int32(world), C.c_int32(rank), C.cast(uid, C.c_void_p),
              C.c_int64(len(uid)), C.byref(comm))

    d, tokens = 768, 20000
    x = torch.randn(tokens, d, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(dev)
    r0, r1 = token_shard(tokens, world, rank)
    part = HessianAccumulator(d, dev)
    part.update(x[r0:r1])
    full = HessianAccumulator(d, dev)
    full.update(x)
    ref = full.get_hessian()

    _lib.call("llmc_hessian_allreduce", C.c_void_p(part._h), comm)
    got = part.get_hessian()
    err = float((got.double() - ref.double()).norm() / ref.double().norm())
    ok = part.sample_count == tokens and err < 1e-5
    print(f"rank {rank}: allreduce rel err {err:.3e}, samples {part.sample_count}", flush=True)

    part.reset()
    part.update(x[r0:r1])
    _lib.call("llmc_hessian_reduce", C.c_void_p(part._h), comm, C.c_int32(1))
    if rank == 1:
        got = part.get_hessian()
        err = float((got.double() - ref.double()).norm() / ref.double().norm())
        ok &= part.sample_count == tokens and err < 1e-5
        print(f"rank {rank}: reduce rel err {err:.3e}, samples {part.sample_count}", flush=True)
    else:
        ok &= part.sample_count == r1 - r0
    torch.cuda.synchronize()
    _lib.call("llmc_nccl_comm_destroy", comm)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
