"""Timed CPU baseline of the decode path (TEST/BENCH INFRASTRUCTURE ONLY).

The reference's CPU implementation of Qwen3 decoding is qwen3/reference.py:
transformers' Qwen3ForCausalLM in bf16 with eager attention, greedy,
KV-cached (reference.py:11-45). This module times that model on the host's
cores for a bounded sample of the benchmark workload:

* the model is built with the benchmark's layer shapes and vocabulary, but
  with `sample_layers` (two depths, default 1 and 3) instead of all layers,
  with random bf16 weights (timing does not depend on their values);
* each sample model prefills the benchmark's prompt length in one batched
  forward (as reference.py's generate does) and then times `steps` cached
  one-token decode steps;
* per-token time is fitted as fixed + layers * per_layer from the two depths
  and evaluated at the full depth: tok/s = 1 / (fixed + L * per_layer).

Used by bench.py's cpu_baseline leg and its --impl reference arm.
"""

from __future__ import annotations

import os
import time

from xpu_playground_b200.qwen3_config import HEAD_DIM, Qwen3Shape


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


def _time_depth(shape: Qwen3Shape, layers: int, context: int, steps: int) -> float:
    """Seconds per cached decode step at `context` prompt tokens."""
    import torch

    model = _build(shape, layers)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, shape.vocab, (1, context), generator=g)
    with torch.no_grad():
        out = model(input_ids=ids, use_cache=True, logits_to_keep=1)
        past = out.past_key_values
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        pos = context
        # one untimed step, then the timed ones
        out = model(input_ids=tok, position_ids=torch.tensor([[pos]]), past_key_values=past, use_cache=True)
        past, tok, pos = out.past_key_values, out.logits[:, -1].argmax(-1, keepdim=True), pos + 1
        t0 = time.perf_counter()
        for _ in range(steps):
            out = model(input_ids=tok, position_ids=torch.tensor([[pos]]), past_key_values=past, use_cache=True)
            past, tok, pos = out.past_key_values, out.logits[:, -1].argmax(-1, keepdim=True), pos + 1
        dt = (time.perf_counter() - t0) / steps
    del model, past, out
    return dt


def hf_decode_baseline(shape: Qwen3Shape, context: int, steps: int = 6,
                       sample_layers: tuple[int, int] = (1, 3), threads: int | None = None) -> dict:
    import torch

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    t_start = time.perf_counter()
    l0, l1 = sample_layers
    t0 = _time_depth(shape, l0, context, steps)
    t1 = _time_depth(shape, l1, context, steps)
    per_layer = max((t1 - t0) / (l1 - l0), 0.0)
    fixed = max(t0 - l0 * per_layer, 0.0)
    per_token = fixed + shape.layers * per_layer
    return {
        "value": 1.0 / per_token,
        "unit": "tok/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"transformers Qwen3ForCausalLM bf16 eager (qwen3/reference.py's model) on the host: "
                   f"{l0}- and {l1}-layer models with this shape, {context}-token batched prefill, "
                   f"{steps} timed cached decode steps each; per-token time fitted as fixed + layers * "
                   f"per_layer ({fixed * 1e3:.1f} ms + {shape.layers} x {per_layer * 1e3:.2f} ms) "
                   f"at {shape.layers} layers; {time.perf_counter() - t_start:.0f} s of host time"),
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
