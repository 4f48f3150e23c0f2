#!/usr/bin/env python3
"""Benchmark: Qwen3-8B-shaped greedy decode on B200 (the headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one greedy decode token of a batch-1 Qwen3-8B-shaped model
(36 layers, hidden 4096, 32/8 heads, intermediate 12288, vocabulary 151936,
untied lm_head; seeded synthetic bf16 weights N(0, 0.02), norms 1) after a
2048-token seeded prompt, i.e. BASELINE configs[4] at batch 1.

* value: device-resident decoding (the step's input token is the previous
  step's greedy token, no host round trip), timed with CUDA events around
  exactly K steps on the engine's stream, max over ranks.
* e2e: the same decode through the reference-facing API (xpu_qwen3_decode,
  qwen3/main.cpp Engine::decode): per step a host->device copy of the input
  token/position from pinned memory and a device->host read of the result.
* roofline: the decode step is one persistent kernel per token (k_step), so
  the dominant kernel's achieved bandwidth is its algorithmic bytes per launch
  (every weight once, one embedding row, K/V for the live context) over its
  event-timed duration.
* cpu_baseline / --impl reference: transformers' Qwen3ForCausalLM in bf16
  (qwen3/reference.py's model) on the host cores, bounded sample (see
  oracle/cpu_baseline.py).

Multi-GPU: with torchrun, the N ranks (one per GPU) run ONE N-way
tensor-parallel engine (q/k/v and gate/up sharded by rows, o_proj/down by
canonical K chunks exchanged over NVLink inside the step kernel, lm_head by
vocabulary rows), so `value` is the tok/s of that single sequence and
`scaling` is "strong". The 16384 x 16384 GEMVs in `extra` are row-sharded
over the N ranks (aggregate GB/s over the max-over-ranks time); the GEMMs run
on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Qwen3 decode tok/s @1/2/4/8 B200; GEMV GB/s & GEMM TFLOP/s vs roofline"
FALLBACK_HBM_GBS = 6650.0  # profiling recipe's fallback, used only without MEASURED_PEAKS.json
# dram__bytes_read.sum + dram__bytes_write.sum per launch of k_step divided by
# its algorithmic bytes, measured by ncu on the 8B-shaped 2-layer step
# (2.0334 GB read + 3.6 MB written for 2.0333 GB of algorithmic bytes at a
# 2051-position context); traffic grows with the weights streamed, so the
# ratio carries over to 36 layers.
TRAFFIC_RATIO = 1.002


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--preset", default="qwen3-8b")
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--mode", choices=["persistent", "graph"], default="persistent")
    ap.add_argument("--e2e-steps", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv", action="store_true")
    ap.add_argument("--no-small", action="store_true", help="skip the Qwen3-0.6B decode measurement in extra")
    ap.add_argument("--batch", type=int, default=16,
                    help="sequences of the batched-decode measurement in extra (0: skip)")
    ap.add_argument("--record-tokens", metavar="PATH",
                    help="write this run's greedy tokens as the stored run the token check compares with")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str | None):
        self.uuid = device_uuid
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if self.uuid:
            cmd.insert(1, f"--id={self.uuid}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.send_signal(signal.SIGTERM)
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
            os.unlink(self.path)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def seeded_prompt(n: int, vocab: int, seed: int = 7) -> list[int]:
    import numpy as np
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, size=n)]


def row_shard(m: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of an m-row matrix that rank `rank` of `world` holds."""
    return m * rank // world, m * (rank + 1) // world


def gemv_extra(torch, device, rank: int = 0, world: int = 1) -> dict:
    """GEMV GB/s at BASELINE configs[0]/[1] shapes (seeded uniform inputs,
    matrix read once per launch, inputs rotated so nothing stays in L2). With
    world > 1 the 16384 x 16384 matrices are row-sharded: rank r holds rows
    [r M / world, (r + 1) M / world) of the one seeded matrix, and GB/s is
    the whole matrix over the max-over-ranks time; the 4096 x 4096 GEMV stays
    on rank 0."""
    import torch.distributed as dist

    from xpu_playground_b200 import _lib, kernels
    L = _lib.load()
    out = {}
    for name, m, k, dt, code in (("gemv_4096_bf16", 4096, 4096, torch.bfloat16, _lib.XPU_BF16),
                                 ("gemv_16384_bf16", 16384, 16384, torch.bfloat16, _lib.XPU_BF16),
                                 ("gemv_16384_fp16", 16384, 16384, torch.float16, _lib.XPU_FP16)):
        sharded = world > 1 and m == 16384
        if world > 1 and not sharded and rank != 0:
            continue
        m_full = m
        r0, r1 = row_shard(m_full, world, rank) if sharded else (0, m_full)
        m = r1 - r0
        copies = max(1, (512 << 20) // (2 * m * k))  # > L2 worth of matrices, used round-robin
        mats = []
        for c in range(copies):
            # every rank fills the whole seeded matrix and keeps a view of its
            # rows, so the shards are the rows of one matrix at every N
            full = torch.empty(m_full, k, dtype=dt, device=device)
            _lib.check(L.xpu_fill_uniform16(code, full.data_ptr(), m_full * k, 11 + c, 1, None))
            mats.append(full[r0:r1])
        x = torch.empty(k, dtype=dt, device=device)
        _lib.check(L.xpu_fill_uniform16(code, x.data_ptr(), k, 12, 2, None))
        y = torch.empty(m, dtype=dt, device=device)
        for i in range(5):
            kernels.gemv(mats[i % copies], x, y)
        # 50 launches (matrices round-robin) captured in a CUDA graph and
        # timed with events around one replay: device time per launch,
        # without the host's per-call overhead (a 4096^2 launch streams
        # 32 MiB in a few microseconds, less than one Python call).
        reps = 50
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(reps):
                kernels.gemv(mats[i % copies], x, y)
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        sec = e0.elapsed_time(e1) * 1e-3 / reps
        del graph
        if sharded:
            t = torch.tensor([sec], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t.item())
        out[name] = {"GB/s": round(2 * m_full * k / sec / 1e9, 1), "us": round(sec * 1e6, 2),
                     "timing": "CUDA graph of 50 launches, matrices rotated past L2"}
        if sharded:
            out[name]["row_shards"] = world
        del mats
    return out


def gemm_extra(torch, device, peak_tflops: float) -> dict:
    """GEMM TFLOP/s at BASELINE configs[2] shapes (seeded uniform[-1, 1]
    operands; 5 warm-up launches, then 20 back-to-back launches timed with
    CUDA events; operands are L2-resident, the kernel is tensor-bound), and
    beside each the vendor library on the same operands and shape
    (torch.matmul, i.e. cuBLAS), timed the same way."""
    from xpu_playground_b200 import _lib, kernels
    L = _lib.load()
    out = {}
    for name, (m, n, k), dt, code in (("gemm_4096_bf16", (4096, 4096, 4096), torch.bfloat16, _lib.XPU_BF16),
                                      ("gemm_3072x4096x2048_fp16", (3072, 4096, 2048), torch.float16,
                                       _lib.XPU_FP16)):
        A = torch.empty(m, k, dtype=dt, device=device)
        B = torch.empty(k, n, dtype=dt, device=device)
        C = torch.empty(m, n, dtype=dt, device=device)
        _lib.check(L.xpu_fill_uniform16(code, A.data_ptr(), m * k, 21, 1, None))
        _lib.check(L.xpu_fill_uniform16(code, B.data_ptr(), k * n, 21, 2, None))
        for _ in range(5):
            kernels.gemm(A, B, C)
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            kernels.gemm(A, B, C)
        e1.record()
        e1.synchronize()
        sec = e0.elapsed_time(e1) * 1e-3 / reps
        tf = 2.0 * m * n * k / sec / 1e12
        if kernels.device_status():
            raise SystemExit("GEMM device error")
        C2 = torch.empty_like(C)
        for _ in range(5):
            torch.matmul(A, B, out=C2)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            torch.matmul(A, B, out=C2)
        e1.record()
        e1.synchronize()
        sec_lib = e0.elapsed_time(e1) * 1e-3 / reps
        tf_lib = 2.0 * m * n * k / sec_lib / 1e12
        out[name] = {"TFLOP/s": round(tf, 1), "us": round(sec * 1e6, 2),
                     "frac_of_measured_bf16_peak": round(tf / peak_tflops, 4),
                     "cublas": {"TFLOP/s": round(tf_lib, 1), "us": round(sec_lib * 1e6, 2),
                                "call": "torch.matmul on the same operands"},
                     "vs_cublas": round(tf / tf_lib, 4)}
        del A, B, C, C2
    return out


def batch_extra(torch, device, shape, context: int, batch: int, steps: int, warmup: int,
                rank: int = 0, world: int = 1, group=None) -> dict:
    """Batched decode (BASELINE configs[4] at batch 16): `batch` sequences,
    each after its own seeded `context`-token prompt (prefilled by batched
    steps), timed over `steps` device-resident batched steps with CUDA
    events (max over ranks; tensor parallel over the ranks at N > 1);
    roofline = this GPU's weights once + every sequence's K/V per step."""
    from xpu_playground_b200.qwen3 import Qwen3Engine

    max_seq = context + warmup + steps + 8
    eng = Qwen3Engine(shape, max_seq, device=device.index or 0, tp_rank=rank, tp_size=world, max_batch=batch)
    eng.init_synthetic(WEIGHT_SEED)
    if world > 1:
        eng.connect_tensor_parallel(group)
    prompts = [seeded_prompt(context, shape.vocab, seed=7 + s) for s in range(batch)]
    eng.batch_generate(prompts, 1)  # prefill: context batched steps
    stream = torch.cuda.ExternalStream(eng.info().stream, device=device)
    eng.batch_enqueue_steps(warmup)
    eng.synchronize()
    _, pos0, err = eng.batch_state(batch)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eng.batch_enqueue_steps(steps)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    _, pos1, err = eng.batch_state(batch)
    if err:
        raise RuntimeError(f"batched decode error word {err}")
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    mid = (pos0[0] + pos1[0]) // 2
    nbytes = eng.batch_bytes_per_step(batch, mid)
    peak, kind = measured_peaks()
    out = {
        "workload": f"{shape.layers}-layer {shape.hidden}-hidden greedy decode, batch {batch}, "
                    f"{context}-token prompt per sequence",
        "value": round(batch * 1000.0 / ms, 1), "unit": "tok/s", "ms_per_step": round(ms, 4),
        "steps": steps, "context_tokens": [pos0[0], pos1[0]], "n_gpus": world,
        "kernels_per_step": eng.batch_kernels_per_step(),
        "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": nbytes,
                     "achieved": round(nbytes / (ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
                     "peak_source": f"{kind} HBM copy bandwidth"},
    }
    eng.close()
    return out


def small_extra(torch, device, warmup: int) -> dict:
    """the Qwen3-0.6B shape (28 layers, hidden 1024,
    16/8 heads, tied), a 128-token seeded prompt (chunked prefill), then 128
    device-resident greedy decode steps timed with CUDA events; roofline =
    every weight once + the live K/V per step. At 1.2 GB per token the step is
    bound by its per-layer phase latencies rather than by HBM."""
    from xpu_playground_b200.qwen3 import Qwen3Engine
    from xpu_playground_b200.qwen3_config import PRESETS

    shape, prompt_len, steps = PRESETS["qwen3-0.6b"], 128, 128
    eng = Qwen3Engine(shape, prompt_len + warmup + steps + 8, device=device.index or 0)
    eng.init_synthetic(WEIGHT_SEED)
    eng.prefill(seeded_prompt(prompt_len, shape.vocab))
    stream = torch.cuda.ExternalStream(eng.info().stream, device=device)
    eng.enqueue_steps(warmup)
    eng.synchronize()
    _, pos0, _ = eng.state()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eng.enqueue_steps(steps)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    _, pos1, err = eng.state()
    if err:
        raise SystemExit(f"0.6B decode error word {err}")
    nbytes = eng.bytes_per_token((pos0 + pos1) // 2)
    peak, kind = measured_peaks()
    eng.close()
    return {"workload": "qwen3-0.6b-shaped greedy decode, batch 1, 128-token prompt then 128 decode steps",
            "value": round(1000.0 / ms, 1), "unit": "tok/s", "ms_per_step": round(ms, 4),
            "context_tokens": [pos0, pos1],
            "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": nbytes,
                         "achieved": round(nbytes / (ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
                         "peak_source": f"{kind} HBM copy bandwidth"}}


def measured_tflops() -> float:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except Exception:
        return 1590.0  # profiling recipe's fallback burst figure


def decode_config(args, shape) -> dict:
    """The workload both arms report, identically (the reference arm times
    the same model shape and prompt length on the host)."""
    return {"workload": f"{args.preset}-shaped greedy decode, batch 1, {args.context}-token prompt then "
                        f"{args.steps} timed decode steps",
            "layers": shape.layers, "hidden": shape.hidden, "heads": f"{shape.q_heads}/{shape.kv_heads}",
            "intermediate": shape.intermediate, "vocab": shape.vocab, "tied_lm_head": shape.tied,
            "context": args.context,
            "l2": "inputs larger than L2: each step streams all weights (15.4 GB for the 8B shape) once"}


WEIGHT_SEED = 2026
GOLDEN_TOKENS = ROOT / "tests" / "golden" / "decode_tokens_qwen3-8b.json"
PREFILL_PATH = "xpu_qwen3_prefill_dense"  # the prefill the checked decode continues from


def token_digest(ids: list[int]) -> str:
    import hashlib
    import struct
    return hashlib.sha256(struct.pack(f"<{len(ids)}I", *ids)).hexdigest()


def check_tokens(args, first: int, ids: list[int]) -> dict:
    """The run's greedy tokens against the stored one-GPU run of the same
    weights seed, prompt and prefill (tests/golden/decode_tokens_qwen3-8b.json,
    written by `bench.py --record-tokens` on one GPU): the common prefix must
    be identical."""
    info = {"first_position": first, "count": len(ids), "sha256": token_digest(ids), "ids": ids,
            "prefill": PREFILL_PATH + ", at every N"}
    try:
        gold = json.loads(GOLDEN_TOKENS.read_text())
    except (OSError, ValueError):
        info["golden"] = None
        return info
    same_run = (gold.get("preset") == args.preset and gold.get("context") == args.context and
                gold.get("weight_seed") == WEIGHT_SEED and gold.get("first_position") == first and
                gold.get("prefill") == PREFILL_PATH)
    if not same_run:
        info["golden"] = None
        return info
    n = min(len(ids), len(gold["ids"]))
    info["golden"] = {"file": str(GOLDEN_TOKENS.relative_to(ROOT)), "n_gpus": gold.get("n_gpus"),
                      "compared": n, "sha256_of_compared": token_digest(gold["ids"][:n]),
                      "match": ids[:n] == gold["ids"][:n]}
    return info


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from xpu_playground_b200.qwen3 import Qwen3Engine
    from xpu_playground_b200.qwen3_config import PRESETS

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    shape = PRESETS[args.preset]
    K, W, E = args.steps, args.warmup, args.e2e_steps
    max_seq = args.context + W + K + E + 8
    mode = args.mode if world == 1 else "persistent"  # tensor parallel runs the persistent step
    eng = Qwen3Engine(shape, max_seq, device=local, tp_rank=rank, tp_size=world, mode=mode)
    eng.init_synthetic(WEIGHT_SEED)
    tp_group = None
    if world > 1:
        tp_group = dist.new_group(backend="gloo")
        eng.connect_tensor_parallel(tp_group)
    prompt = seeded_prompt(args.context, shape.vocab)
    chunked = None
    if world == 1:
        # The 16-positions-per-step chunked prefill, for comparison (one GPU;
        # synchronous, host wall clock); the dense prefill below replaces its
        # KV cache.
        eng.synchronize()
        t_pre = time.perf_counter()
        eng.prefill(prompt)
        t_chunk = time.perf_counter() - t_pre
        chunked = {"seconds": round(t_chunk, 4), "tok_s": round(args.context / t_chunk, 1),
                   "positions_per_step": 16, "path": "xpu_qwen3_prefill"}
    # Dense prefill at every N (every position through each layer together,
    # tcgen05 GEMMs against the stored weights; under tensor parallelism the
    # row-parallel sums cross NVLink): one untimed call, then the timed one,
    # host wall clock around the synchronous call, max over ranks. The timed
    # decode continues from its KV cache, and the dense prefill computes the
    # same bits at every tensor-parallel size, so the greedy tokens compared
    # across GPU counts cover prefill and decode.
    eng.synchronize()
    eng.prefill_dense(prompt)
    if world > 1:
        dist.barrier()
    t_pre = time.perf_counter()
    eng.prefill_dense(prompt)
    t_dense = time.perf_counter() - t_pre
    if world > 1:
        t = torch.tensor([t_dense], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_dense = float(t.item())
    prefill_info = {"tokens": args.context, "seconds": round(t_dense, 4), "tok_s": round(args.context / t_dense, 1),
                    "path": PREFILL_PATH, "n_gpus": world,
                    "timing": "host wall clock around the synchronous call (prompt upload and token read included)"}
    if chunked:
        prefill_info["chunked"] = chunked
    stream = torch.cuda.ExternalStream(eng.info().stream, device=device)
    eng.enqueue_steps(W)
    eng.synchronize()
    _, pos0, err = eng.state()
    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(device)
    uuid = str(getattr(props, "uuid", "") or "")
    clocks = ClockSampler(("GPU-" + uuid) if uuid and not uuid.startswith("GPU-") else (uuid or None))
    clocks.start()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eng.enqueue_steps(K)
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize(device)
    clock_info = clocks.stop()
    ms = e0.elapsed_time(e1) / K
    tok, pos1, err = eng.state()
    if err:
        raise SystemExit(f"decode error word {err}")
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()

    # e2e through the reference-facing API: host token in, host token out.
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nxt = tok
    f0.record(stream)
    for i in range(E):
        nxt = eng.decode(nxt, pos1 + i)
    f1.record(stream)
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1) / E
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    first = args.context - 1  # the prompt's last position holds the first generated token
    tokens = check_tokens(args, first, eng.token_log(first, pos1 + E - first))
    if args.record_tokens and rank == 0:
        Path(args.record_tokens).write_text(json.dumps(
            {"preset": args.preset, "context": args.context, "weight_seed": WEIGHT_SEED,
             "prompt": "bench.seeded_prompt(context, vocab) (numpy default_rng(7))", "prefill": PREFILL_PATH,
             "n_gpus": world,
             "first_position": first, "ids": tokens["ids"], "sha256": tokens["sha256"]}) + "\n")

    mid_context = (pos0 + pos1) // 2
    bytes_step = eng.bytes_per_token(mid_context)
    achieved = bytes_step / (ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()

    extra = {}
    if prefill_info:
        extra["prefill"] = prefill_info
    if not args.no_small and world == 1:
        eng.synchronize()
        extra["qwen3_0p6b_decode"] = small_extra(torch, device, warmup=max(W, 3))
    if args.batch:
        eng.synchronize()
        try:
            extra["batch_decode"] = batch_extra(torch, device, shape, args.context, args.batch,
                                                steps=min(K, 64), warmup=max(W, 3), rank=rank, world=world,
                                                group=tp_group)
        except Exception as e:  # recorded in the line; the headline stands on its own
            extra["batch_decode"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if not args.no_gemv:
        eng.synchronize()
        extra.update(gemv_extra(torch, device, rank, world))
        if rank == 0:
            extra.update(gemm_extra(torch, device, measured_tflops()))
    launches = K * eng.info().kernels_per_step
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    # The host-core baselines run on rank 0 after every GPU rank is done, on
    # the threads this process may use.
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as orc
        from oracle.cpu_baseline import gemm_cpu_baseline, gemv_cpu_baseline, hf_decode_baseline, host_threads
        orc.set_threads(host_threads())
        for key, (m, k) in (("gemv_4096_bf16", (4096, 4096)), ("gemv_16384_bf16", (16384, 16384))):
            if key in extra:
                extra[key]["cpu_baseline"] = gemv_cpu_baseline(m, k)
        if "gemm_4096_bf16" in extra:
            extra["gemm_4096_bf16"]["cpu_baseline"] = gemm_cpu_baseline(4096, 4096, 4096)
        cpu = hf_decode_baseline(shape, args.context)
        cpu.pop("per_token_s", None)
        cpu["value"] = round(cpu["value"], 3)

    value = 1000.0 / ms
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) bf16 weights, seeded uniform prompt ids)",
        "config": decode_config(args, shape),
        "run": {
            "context_tokens": [pos0, pos1],
            "decode_mode": mode,
            "parallelism": "single GPU" if world == 1 else f"tp{world} (tensor parallel, one sequence)",
        },
        "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 24,
                "d2h_bytes_per_step": 32},
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": round(TRAFFIC_RATIO * bytes_step) if TRAFFIC_RATIO else None,
            "kernel": "k_step (persistent decode step)" if mode == "persistent" else "decode graph",
            "algorithmic_bytes_per_launch": bytes_step,
            "peak_source": f"{peak_kind} HBM copy bandwidth",
        },
        "cpu_baseline": cpu,
        "clocks": clock_info,
        "gpu_launches": launches,
        "tokens": tokens,
        "extra": extra,
    }
    print(json.dumps(line), flush=True)
    if tokens.get("golden") and not tokens["golden"]["match"]:
        sys.exit(f"greedy tokens differ from the stored one-GPU run ({tokens['golden']['file']})")


def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle.cpu_baseline import hf_decode_baseline
    from xpu_playground_b200.qwen3_config import PRESETS

    shape = PRESETS[args.preset]
    t0 = time.time()
    cpu = hf_decode_baseline(shape, args.context)
    value = cpu["value"]
    cpu.pop("per_token_s", None)
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": round(value, 3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1000.0 / value, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) bf16 weights, seeded uniform prompt ids)",
        "config": decode_config(args, shape),
        "run": {"parallelism": "host CPU (rank 0 alone)"},
        "cpu_baseline": dict(cpu, value=round(value, 3)),
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(time.time() - t0, 1),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
