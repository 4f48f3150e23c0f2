"""Row-sharded GEMV (the multi-GPU GEMV of BASELINE configs[1]): rank r of N
holds rows [r M / N, (r + 1) M / N) of one seeded matrix, computes its part
of y = A.x with no exchange, and the parts gathered in rank order are y.

* CPU (gloo, 2 ranks): the sharding and gather logic with the FP32 host
  loop (gemv.cpp:126-130 restated) standing in for the kernel - the gathered
  y equals the oracle's unsharded y bit for bit.
* GPU (NCCL, 2 ranks on 2 GPUs): xpu_gemv on each rank's rows of the 16384^2
  bf16 matrix; the gathered y is bit-identical to one GPU's unsharded y and
  within 1e-2 relative Frobenius of the FP32 host loop."""

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard(m, world, rank):
    sys.path.insert(0, str(ROOT))
    import bench
    return bench.row_shard(m, world, rank)


def _cpu_rank(rank, world, port, m, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from oracle import oracle as orc
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        A = orc.uniform16(m * k, 11, 1).reshape(m, k)
        x = orc.uniform16(k, 12, 2)
        r0, r1 = _shard(m, world, rank)
        part = orc.gemv(A[r0:r1], x)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        q.put((rank, np.concatenate(parts)))
    finally:
        dist.destroy_process_group()


def test_row_sharded_gemv_two_gloo_ranks():
    from oracle import oracle as orc
    m, k = 1000, 520
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank, args=(r, 2, port, m, k, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    A = orc.uniform16(m * k, 11, 1).reshape(m, k)
    x = orc.uniform16(k, 12, 2)
    want = orc.gemv(A, x)
    for rank in (0, 1):
        assert np.array_equal(results[rank], want)


def _gpu_rank(rank, world, port, m, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from xpu_playground_b200 import _lib, kernels
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        L = _lib.load()
        A = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
        x = torch.empty(k, dtype=torch.bfloat16, device="cuda")
        _lib.check(L.xpu_fill_uniform16(_lib.XPU_BF16, A.data_ptr(), m * k, 11, 1, None))
        _lib.check(L.xpu_fill_uniform16(_lib.XPU_BF16, x.data_ptr(), k, 12, 2, None))
        r0, r1 = _shard(m, world, rank)
        part = kernels.gemv(A[r0:r1], x)
        parts = [torch.empty(_shard(m, world, r)[1] - _shard(m, world, r)[0], dtype=torch.bfloat16, device="cuda")
                 for r in range(world)]
        dist.all_gather(parts, part)
        y = torch.cat(parts)
        whole = kernels.gemv(A, x) if rank == 0 else None
        torch.cuda.synchronize()
        q.put((rank, y.view(torch.int16).cpu().numpy().view(np.uint16),
               None if whole is None else whole.view(torch.int16).cpu().numpy().view(np.uint16)))
        dist.barrier()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
def test_row_sharded_gemv_16384_on_two_gpus():
    from oracle import oracle as orc
    m = k = 16384
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank, args=(r, 2, port, m, k, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = {}
        for _ in procs:
            rank, y, whole = q.get(timeout=600)
            assert not isinstance(y, str), y
            results[rank] = (y, whole)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    y0, whole = results[0]
    assert np.array_equal(y0, results[1][0])
    assert np.array_equal(y0, whole)  # sharding changes no bit of y
    A = orc.uniform16(m * k, 11, 1).reshape(m, k)
    x = orc.uniform16(k, 12, 2)
    assert orc.rel_frobenius(orc.bf16_to_float(y0), orc.gemv(A, x)) < 1e-2
