"""Generate the golden fixtures under tests/golden/ (run in the build container).

Each fixture is produced by the reference's own code or its model oracle,
never by this repository's CUDA library:

* ref_codec.npz      - qwen3/model.cpp float_to_bf16 (compiled in place into
                       oracle/_ref/libref_model.so) on edge-case and random floats.
* hf_rope.npz        - transformers Qwen3RotaryEmbedding cos/sin (bf16 bits) at
                       selected positions up to 40959, theta 1e6, head_dim 128.
* hf_<shape>.npz     - qwen3/reference.py's model (transformers Qwen3ForCausalLM,
                       bf16, eager attention) built from a seeded synthetic
                       checkpoint, decoded token by token: per-step greedy ids
                       and logits (full for small vocabularies, top-64 plus
                       three full steps for the 151936-token vocabulary).

    PYTHONPATH=. python tests/golden/make_golden.py [--only NAME ...]
"""

from __future__ import annotations

import argparse
import ctypes
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import build as oracle_build  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from oracle.qwen3_ref import HFDecoder, hf_version, prompt_ids, seeded_weights  # noqa: E402
from xpu_playground_b200.qwen3_config import PRESETS  # noqa: E402

# (shape preset, weight seed, prompt seed, prompt length, decode steps)
MODEL_CASES = {
    "tiny": ("tiny", 1234, 7, 8, 24),
    "tiny-tied": ("tiny-tied", 99, 11, 12, 20),
    "qwen3-0.6b": ("qwen3-0.6b", 2026, 3, 128, 128),
    "qwen3-8b-l2": ("qwen3-8b-l2", 8, 5, 16, 16),
}


def make_codec() -> None:
    oracle_build.build_reference()
    lib = ctypes.CDLL(str(oracle_build.REF_OUT / "libref_model.so"))
    lib.ref_float_to_bf16.restype, lib.ref_float_to_bf16.argtypes = ctypes.c_uint16, [ctypes.c_float]
    rng = np.random.default_rng(0)
    special = np.array([0.0, -0.0, 1.0, -1.0, 0.1, 100.0, 65504.0, 3.0e38, -3.0e38, 1e-40, -1e-40,
                        np.inf, -np.inf, 1.00390625, 1.01171875, 1.0078125 + 2**-16,
                        np.float32(1.0 + 2**-8), np.float32(1.0 + 3 * 2**-8)], np.float32)
    bits = rng.integers(0, 2**32, size=20000, dtype=np.uint64).astype(np.uint32)
    rand = bits.view(np.float32)
    rand = rand[np.isfinite(rand)]
    inputs = np.concatenate([special, rand, rng.standard_normal(5000).astype(np.float32)])
    outputs = np.array([lib.ref_float_to_bf16(float(v)) for v in inputs], np.uint16)
    np.savez_compressed(HERE / "ref_codec.npz", inputs=inputs, bf16=outputs)


def make_rope() -> None:
    import torch
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    cfg = Qwen3Config(head_dim=128, rope_theta=1e6, max_position_embeddings=40960)
    rot = Qwen3RotaryEmbedding(config=cfg)
    positions = np.array(sorted(set(list(range(0, 64)) + list(range(1000, 1032)) +
                                list(range(2040, 2310, 9)) + list(range(40900, 40960)))), np.int64)
    x = torch.zeros(1, 1, 128, dtype=torch.bfloat16)
    cos, sin = rot(x, torch.from_numpy(positions)[None])
    to_bits = lambda t: t[0].contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    np.savez_compressed(HERE / "hf_rope.npz", positions=positions, cos=to_bits(cos),
                        sin=to_bits(sin), transformers=hf_version())


def make_model(name: str) -> None:
    preset, wseed, pseed, n_prompt, n_decode = MODEL_CASES[name]
    shape = PRESETS[preset]
    t0 = time.time()
    weights = seeded_weights(shape, wseed)
    dec = HFDecoder(shape, weights)
    prompt = prompt_ids(n_prompt, shape.vocab, pseed)
    ids, logits_steps, top_idx, top_val = [], [], [], []
    token = prompt[0]
    full_steps = {0, n_prompt, n_prompt + n_decode - 1}
    for pos in range(n_prompt + n_decode):
        token_in = prompt[pos] if pos < n_prompt else token
        nxt, bits = dec.step(token_in, pos)
        ids.append(nxt)
        if shape.vocab <= 8192:
            logits_steps.append(bits)
        else:
            vals = orc.bf16_to_float(bits)
            order = np.argsort(-vals, kind="stable")[:64]
            top_idx.append(order.astype(np.int32))
            top_val.append(bits[order])
            if pos in full_steps:
                logits_steps.append(bits)
        token = nxt
    extra = {}
    if top_idx:
        extra = dict(top_idx=np.stack(top_idx), top_bits=np.stack(top_val),
                     full_steps=np.array(sorted(full_steps), np.int32))
    np.savez_compressed(HERE / f"hf_{name.replace('.', 'p')}.npz", preset=preset, weight_seed=wseed,
                        prompt=np.array(prompt, np.int32), steps=n_prompt + n_decode,
                        greedy=np.array(ids, np.int32), logits=np.stack(logits_steps),
                        transformers=hf_version(), **extra)
    print(f"{name}: {n_prompt}+{n_decode} steps in {time.time() - t0:.1f}s")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*", default=None)
    args = ap.parse_args()
    todo = args.only or ["codec", "rope", *MODEL_CASES]
    if "codec" in todo:
        make_codec()
    if "rope" in todo:
        make_rope()
    for name in MODEL_CASES:
        if name in todo:
            make_model(name)


if __name__ == "__main__":
    main()
