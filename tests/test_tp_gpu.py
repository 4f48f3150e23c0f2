"""Tensor-parallel decode on 2, 4 and 8 GPUs (one process per GPU, gloo for
the host rendezvous, NVLink peer stores for the exchange): every tp_size
gives the same greedy tokens and bit-identical logits as one GPU, and a rank
that never joins a step makes its peers' bounded waits end with
XPU_ERR_TIMEOUT instead of a hang."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.qwen3_ref import prompt_ids
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
SEED = 11
MAX_SEQ = 256


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_generate(rank, world, port, preset, prompt, n_new, q, ckpt=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        eng = Qwen3Engine(PRESETS[preset], MAX_SEQ, device=rank, tp_rank=rank, tp_size=world)
        if ckpt:
            eng.load_checkpoint(ckpt)  # each rank streams its own shards from the files
        else:
            eng.init_synthetic(SEED)
        eng.connect_tensor_parallel()
        toks = eng.generate(prompt, n_new)
        q.put((rank, toks, eng.logits()))
        dist.barrier()
        eng.close()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


def _run_ranks(target, world, *args, **kwargs):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q), kwargs=kwargs) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = {}
        for _ in procs:
            rank, a, b = q.get(timeout=600)
            results[rank] = (a, b)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    return results


def _single_gpu(preset, prompt, n_new):
    with Qwen3Engine(PRESETS[preset], MAX_SEQ, device=0) as eng:
        eng.init_synthetic(SEED)
        return eng.generate(prompt, n_new), eng.logits()


@pytest.mark.parametrize("preset,world", [("tiny", 2), ("qwen3-0.6b", 2), ("qwen3-8b-l2", 2),
                                          ("qwen3-0.6b", 4), ("qwen3-8b-l2", 4), ("qwen3-8b-l2", 8)])
def test_tp_matches_single_gpu(preset, world):
    if NGPU < world:
        pytest.skip(f"needs {world} GPUs")
    shape = PRESETS[preset]
    prompt = prompt_ids(24, shape.vocab, seed=5)
    n_new = 24
    ref_toks, ref_logits = _single_gpu(preset, prompt, n_new)
    results = _run_ranks(_rank_generate, world, preset, prompt, n_new)
    shard = shape.vocab // world
    for rank in range(world):
        toks, logits = results[rank]
        assert not isinstance(toks, str), toks
        assert toks == ref_toks, f"rank {rank} tokens differ from tp=1"
        assert np.array_equal(logits, ref_logits[rank * shard:(rank + 1) * shard]), f"rank {rank} logits differ"


def _prefill_then_decode(eng, prompt, n_new):
    """Dense prefill of the prompt, then n_new - 1 host-driven decode steps:
    the greedy tokens, the prefill's last-position logits and the last
    step's logits."""
    toks = [eng.prefill_dense(prompt)]
    first_logits = eng.logits()
    for i in range(n_new - 1):
        toks.append(eng.decode(toks[-1], len(prompt) + i))
    return toks, first_logits, eng.logits()


def _rank_prefill(rank, world, port, preset, prompt, n_new, max_seq, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        eng = Qwen3Engine(PRESETS[preset], max_seq, device=rank, tp_rank=rank, tp_size=world)
        eng.init_synthetic(SEED)
        eng.connect_tensor_parallel()
        eng.prefill_dense(prompt[:7])  # an earlier prompt: the exchange epochs carry on across calls
        q.put((rank, _prefill_then_decode(eng, prompt, n_new), None))
        dist.barrier()
        eng.close()
    except Exception as e:
        q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("preset,world,plen", [("tiny", 2, 50), ("tiny", 2, 2100), ("qwen3-8b-l2", 2, 300),
                                               ("qwen3-0.6b", 4, 129), ("qwen3-8b-l2", 4, 300),
                                               ("qwen3-8b-l2", 8, 300)])
def test_tp_dense_prefill_matches_single_gpu(preset, world, plen):
    """Dense prefill under tensor parallelism (row-parallel subtree sums and
    normalised rows exchanged over NVLink) computes the same bits as one GPU:
    the greedy token after the prompt, the prompt's last logits, and the
    decode steps that continue from the KV cache it wrote. 2100 positions
    take two segments."""
    if NGPU < world:
        pytest.skip(f"needs {world} GPUs")
    shape = PRESETS[preset]
    prompt = prompt_ids(plen, shape.vocab, seed=9)
    n_new, max_seq = 12, plen + 16
    with Qwen3Engine(shape, max_seq, device=0) as eng:
        eng.init_synthetic(SEED)
        ref_toks, ref_first, ref_last = _prefill_then_decode(eng, prompt, n_new)
    results = _run_ranks(_rank_prefill, world, preset, prompt, n_new, max_seq)
    shard = shape.vocab // world
    for rank in range(world):
        got, _ = results[rank]
        assert not isinstance(got, str), got
        toks, first, last = got
        assert toks == ref_toks, f"rank {rank} tokens differ from tp=1"
        part = slice(rank * shard, (rank + 1) * shard)
        assert np.array_equal(first, ref_first[part]), f"rank {rank} prefill logits differ"
        assert np.array_equal(last, ref_last[part]), f"rank {rank} decode logits differ"


BATCH_SEQS, BATCH_STEPS = 4, 20


def _batch_streams(vocab):
    return [prompt_ids(BATCH_STEPS, vocab, seed=30 + s) for s in range(BATCH_SEQS)]


def _batch_run(eng, streams, shard):
    """Teacher-forced batched steps: at step t sequence s reads streams[s][t]
    at position t + s (different positions per sequence). Returns every
    step's greedy tokens and logits (this rank's shard)."""
    toks, logits = [], []
    for t in range(BATCH_STEPS):
        toks.append(eng.batch_decode([streams[s][t] for s in range(BATCH_SEQS)],
                                     [t + s for s in range(BATCH_SEQS)]))
        logits.append(np.stack([eng.batch_logits(s)[:shard] for s in range(BATCH_SEQS)]))
    return toks, logits


def _rank_batch(rank, world, port, preset, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        shape = PRESETS[preset]
        eng = Qwen3Engine(shape, MAX_SEQ, device=rank, tp_rank=rank, tp_size=world, max_batch=BATCH_SEQS)
        eng.init_synthetic(SEED)
        eng.connect_tensor_parallel()
        q.put((rank, _batch_run(eng, _batch_streams(shape.vocab), shape.vocab // world), None))
        dist.barrier()
        eng.close()
    except Exception as e:
        q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("preset,world", [("tiny", 2), ("qwen3-8b-l2", 2), ("qwen3-0.6b", 4), ("qwen3-8b-l2", 8)])
def test_tp_batched_decode_matches_single_gpu(preset, world):
    """Batched decode (4 sequences, each at its own position) under tensor
    parallelism against the one-GPU batched engine on the same inputs: the
    row-parallel partials are summed in rank order rather than in one
    GPU's order, so every step's logits must agree within the full-logit
    gates of the fixture tests, and the greedy tokens must be equal except
    where one GPU's top two logits are within two bf16 steps."""
    if NGPU < world:
        pytest.skip(f"needs {world} GPUs")
    from tests.test_engine_gpu import FULL_MAXABS, FULL_MEANABS, near_tie
    shape = PRESETS[preset]
    streams = _batch_streams(shape.vocab)
    with Qwen3Engine(shape, MAX_SEQ, device=0, max_batch=BATCH_SEQS) as eng:
        eng.init_synthetic(SEED)
        ref_toks, ref_logits = _batch_run(eng, streams, shape.vocab)
    results = _run_ranks(_rank_batch, world, preset)
    shard = shape.vocab // world
    f = __import__("oracle.oracle", fromlist=["bf16_to_float"]).bf16_to_float
    for rank in range(world):
        got, _ = results[rank]
        assert not isinstance(got, str), got
        toks, logits = got
        for t in range(BATCH_STEPS):
            e = f(ref_logits[t][:, rank * shard:(rank + 1) * shard]).astype(np.float64)
            d = np.abs(f(logits[t]).astype(np.float64) - e)
            assert d.max() <= FULL_MAXABS and d.mean() <= FULL_MEANABS, (rank, t, d.max(), d.mean())
            for s in range(BATCH_SEQS):
                if toks[t][s] != ref_toks[t][s]:
                    assert near_tie(ref_logits[t][s], toks[t][s], ref_toks[t][s]), (rank, t, s)


def test_tp_loads_checkpoint_shards(tmp_path):
    """Each rank streams only its shards of a sharded safetensors checkpoint;
    tp=2 then matches one GPU on the same weights."""
    if NGPU < 2:
        pytest.skip("needs 2 GPUs")
    from oracle.qwen3_ref import seeded_weights
    from tests._ckpt import write_checkpoint
    shape = PRESETS["qwen3-0.6b"]
    d = write_checkpoint(tmp_path / "m", shape, seeded_weights(shape, SEED), shards=2)
    prompt = prompt_ids(16, shape.vocab, seed=6)
    ref_toks, ref_logits = _single_gpu("qwen3-0.6b", prompt, 16)
    results = _run_ranks(_rank_generate, 2, "qwen3-0.6b", prompt, 16, ckpt=str(d))
    shard = shape.vocab // 2
    for rank in range(2):
        toks, logits = results[rank]
        assert not isinstance(toks, str), toks
        assert toks == ref_toks
        assert np.array_equal(logits, ref_logits[rank * shard:(rank + 1) * shard])


def _rank_absent_peer(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from xpu_playground_b200._lib import XpuError
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        eng = Qwen3Engine(PRESETS["tiny"], MAX_SEQ, device=rank, tp_rank=rank, tp_size=world)
        eng.init_synthetic(SEED)
        eng.connect_tensor_parallel()
        outcome = "no-step"
        if rank == 0:  # rank 1 never runs the step: rank 0's exchange waits must run out
            try:
                eng.decode(7, 0)
                outcome = "completed"
            except XpuError as e:
                outcome = f"status {e.status}"
            # the engine refuses to continue after a failed exchange
            try:
                eng.decode(7, 0)
                outcome += ", reused"
            except XpuError as e:
                outcome += f", then status {e.status}"
        dist.barrier()  # rank 1 keeps its region mapped until rank 0 is done
        q.put((rank, outcome, None))
        eng.close()
    finally:
        dist.destroy_process_group()


def test_tp_absent_rank_times_out():
    if NGPU < 2:
        pytest.skip("needs 2 GPUs")
    results = _run_ranks(_rank_absent_peer, 2)
    assert results[0][0] == "status 4, then status 1"  # XPU_ERR_TIMEOUT, then XPU_ERR_INVALID
    assert results[1][0] == "no-step"
