"""Timed CPU baseline of the decode path (TEST/BENCH INFRASTRUCTURE ONLY).

The reference's CPU implementation of Qwen3 decoding is qwen3/reference.py:
transformers' Qwen3ForCausalLM in bf16 with eager attention, greedy,
KV-cached (reference.py:11-45). This module times that model on the host's
cores for a bounded sample of the benchmark workload:

* one model is built with the benchmark's layer shapes and vocabulary and
  the deepest sample depth (default 8 layers), random bf16 weights (timing
  does not depend on their values);
* for each sample depth d (default 1, 2, 4, 8) the model runs its first d
  layers: it prefills the benchmark's prompt length in one batched forward
  (as reference.py's generate does), then times `repeats` runs of `steps`
  cached one-token decode steps; the depth's time is its fastest run (the
  host is shared with other jobs, whose interference only ever adds time);
* per-token time is a least-squares line fixed + d * per_layer through the
  depths, evaluated at the full depth: tok/s = 1 / (fixed + L * per_layer).
  The line's worst relative residual and each depth's repeat spread are
  reported with the value.

The thread count is the host threads this process may run on (its CPU
affinity, capped by a cgroup CPU quota when one is set), stated as `cores`.
Used by bench.py's cpu_baseline leg and its --impl reference arm, with the
same arguments in both.
"""

from __future__ import annotations

import os
import statistics
import time

from xpu_playground_b200.qwen3_config import HEAD_DIM, Qwen3Shape

SAMPLE_DEPTHS = (1, 2, 4, 8)
SAMPLE_STEPS = 16
SAMPLE_REPEATS = 5


def host_threads() -> int:
    """CPUs this process may use: its affinity set, capped by a cgroup v2
    CPU quota (cpu.max) when one is set."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    try:
        quota, period = open("/sys/fs/cgroup/cpu.max").read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def _build(shape: Qwen3Shape, layers: int):
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    cfg = Qwen3Config(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                      num_hidden_layers=layers, num_attention_heads=shape.q_heads,
                      num_key_value_heads=shape.kv_heads, head_dim=HEAD_DIM, vocab_size=shape.vocab,
                      tie_word_embeddings=shape.tied, rms_norm_eps=shape.eps,
                      rope_theta=shape.rope_theta, max_position_embeddings=40960,
                      attn_implementation="eager", torch_dtype="bfloat16")
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
    model = model.to_empty(device="cpu").to(torch.bfloat16)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02)
    if shape.tied:
        model.tie_weights()
    model.model.rotary_emb = Qwen3RotaryEmbedding(config=cfg)
    return model.eval()


def _use_depth(model, layers, layer_types, depth: int) -> None:
    """Make the model run only its first `depth` decoder layers."""
    model.model.layers = layers[:depth]
    model.config.num_hidden_layers = depth
    if layer_types is not None:
        model.config.layer_types = list(layer_types[:depth])


def _time_steps(model, shape: Qwen3Shape, context: int, steps: int, repeats: int) -> list[float]:
    """Seconds per cached decode step after one `context`-token prefill:
    `repeats` consecutive runs of `steps` steps (the context grows by
    `steps` per run, a negligible change at benchmark lengths)."""
    import torch

    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, shape.vocab, (1, context), generator=g)
    runs = []
    with torch.no_grad():
        out = model(input_ids=ids, use_cache=True, logits_to_keep=1)
        past = out.past_key_values
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        pos = context
        # one untimed step, then the timed ones
        out = model(input_ids=tok, position_ids=torch.tensor([[pos]]), past_key_values=past, use_cache=True)
        past, tok, pos = out.past_key_values, out.logits[:, -1].argmax(-1, keepdim=True), pos + 1
        for _ in range(repeats):
            t0 = time.perf_counter()
            for _ in range(steps):
                out = model(input_ids=tok, position_ids=torch.tensor([[pos]]), past_key_values=past,
                            use_cache=True)
                past, tok, pos = out.past_key_values, out.logits[:, -1].argmax(-1, keepdim=True), pos + 1
            runs.append((time.perf_counter() - t0) / steps)
    del past, out
    return runs


def fit_line(points: dict[int, float]) -> tuple[float, float, float]:
    """Least-squares t = fixed + d * per_layer through (d, t); returns
    (fixed, per_layer, worst relative residual)."""
    ds = sorted(points)
    n = len(ds)
    md = sum(ds) / n
    mt = sum(points[d] for d in ds) / n
    sdd = sum((d - md) ** 2 for d in ds)
    per_layer = sum((d - md) * (points[d] - mt) for d in ds) / sdd if sdd else 0.0
    fixed = mt - per_layer * md
    resid = max(abs(fixed + d * per_layer - points[d]) / points[d] for d in ds)
    return fixed, per_layer, resid


def hf_decode_baseline(shape: Qwen3Shape, context: int, steps: int = SAMPLE_STEPS,
                       depths: tuple[int, ...] = SAMPLE_DEPTHS, repeats: int = SAMPLE_REPEATS,
                       threads: int | None = None) -> dict:
    import torch

    threads = threads or host_threads()
    torch.set_num_threads(threads)
    t_start = time.perf_counter()
    model = _build(shape, max(depths))
    layers, layer_types = model.model.layers, getattr(model.config, "layer_types", None)
    best, spreads = {}, {}
    for d in depths:
        _use_depth(model, layers, layer_types, d)
        reps = _time_steps(model, shape, context, steps, repeats)
        best[d] = min(reps)
        spreads[d] = (max(reps) - min(reps)) / statistics.median(reps)
    del model, layers
    fixed, per_layer, resid = fit_line(best)
    per_token = fixed + shape.layers * per_layer
    depth_ms = ", ".join(f"{d}: {best[d] * 1e3:.2f} ms" for d in depths)
    return {
        "value": 1.0 / per_token,
        "unit": "tok/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"transformers Qwen3ForCausalLM bf16 eager (qwen3/reference.py's model) on {threads} host "
                   f"threads: the model's first d layers for d in {list(depths)} (this shape), "
                   f"{context}-token batched prefill, then {repeats} runs of {steps} timed cached decode steps, "
                   f"fastest run per depth ({depth_ms}); per-token time = least-squares fixed + d x per_layer "
                   f"({fixed * 1e3:.2f} ms + {shape.layers} x {per_layer * 1e3:.3f} ms) at {shape.layers} "
                   f"layers; {time.perf_counter() - t_start:.0f} s of host time"),
        "fit": {"fixed_ms": round(fixed * 1e3, 3), "per_layer_ms": round(per_layer * 1e3, 4),
                "worst_residual": round(resid, 4),
                "repeat_spread": {str(d): round(spreads[d], 4) for d in depths}},
        "per_token_s": per_token,
    }


def _timed(fn, min_seconds: float) -> float:
    """Seconds per call of fn after one warm-up call, averaged over repeats
    that together take at least min_seconds."""
    fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            return (time.perf_counter() - t0) / reps


def gemv_cpu_baseline(m: int, k: int, fp16: bool = False, min_seconds: float = 1.0) -> dict:
    """The reference's host GEMV check loop (gemv.cpp:126-130: FP32
    accumulation over decoded 16-bit inputs, row by row), restated as
    orc_gemv and run on every host thread, timed on the benchmark's own shape
    with seeded uniform[-1, 1] inputs; matrix GB/s (2 m k bytes per call)."""
    from oracle import oracle as orc
    A = orc.uniform16(m * k, 5, 1, fp16).reshape(m, k)
    x = orc.uniform16(k, 5, 2, fp16)
    dt = _timed(lambda: orc.gemv(A, x, fp16), min_seconds)
    return {"value": round(2.0 * m * k / dt / 1e9, 2), "unit": "GB/s", "cores": orc.num_threads(),
            "kind": "port", "sample": f"{m}x{k} {'fp16' if fp16 else 'bf16'}, FP32 host loop, "
                                      f"{dt * 1e3:.1f} ms per call"}


def gemm_cpu_baseline(m: int, n: int, k: int, fp16: bool = False, sample_rows: int = 128,
                      min_seconds: float = 1.0) -> dict:
    """FP32 host GEMM (orc_gemm: rows of C across every host thread, each
    accumulating over k in order) on a bounded sample of the benchmark shape:
    `sample_rows` of the m rows of C against the full k x n operand; TFLOP/s
    of the sample (2 rows n k FLOP per call), which a whole m x n x k product
    would take m / sample_rows times as long to reach."""
    from oracle import oracle as orc
    rows = min(sample_rows, m)
    A = orc.uniform16(rows * k, 6, 1, fp16).reshape(rows, k)
    B = orc.uniform16(k * n, 6, 2, fp16).reshape(k, n)
    dt = _timed(lambda: orc.gemm(A, B, fp16), min_seconds)
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 5), "unit": "TFLOP/s", "cores": orc.num_threads(),
            "kind": "port", "sample": f"{rows} of {m} rows of C, n {n}, k {k}, {'fp16' if fp16 else 'bf16'} inputs, "
                                      f"FP32 host loop, {dt:.2f} s per call"}
