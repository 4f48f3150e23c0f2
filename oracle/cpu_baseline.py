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
