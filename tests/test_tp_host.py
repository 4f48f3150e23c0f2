"""Host side of the tensor-parallel rendezvous on CPU: two gloo ranks
all-gather their exchange-region handles in rank order (the step the engines
need before tp_connect)."""

import os
import socket
from datetime import timedelta

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from xpu_playground_b200.qwen3 import exchange_handles
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        handle = bytes([rank + 1]) * 64
        q.put((rank, exchange_handles(handle)))
    finally:
        dist.destroy_process_group()


def test_exchange_handles_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expected = [bytes([1]) * 64, bytes([2]) * 64]
    assert results[0] == expected and results[1] == expected
