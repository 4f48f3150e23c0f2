"""Writes Qwen3 checkpoints in the safetensors layout transformers saves
(config.json, model.safetensors or model-0000k-of-0000n.safetensors + index)
for the loader tests: an 8-byte little-endian header length, the JSON header
(dtype, shape, data_offsets per tensor), then the payloads."""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from xpu_playground_b200.qwen3_config import Qwen3Shape


def config_dict(shape: Qwen3Shape, **overrides) -> dict:
    cfg = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_act": "silu",
        "hidden_size": shape.hidden, "intermediate_size": shape.intermediate,
        "num_hidden_layers": shape.layers, "num_attention_heads": shape.q_heads,
        "num_key_value_heads": shape.kv_heads, "head_dim": 128, "vocab_size": shape.vocab,
        "rms_norm_eps": shape.eps, "rope_theta": shape.rope_theta, "rope_scaling": None,
        "tie_word_embeddings": shape.tied, "torch_dtype": "bfloat16",
        "max_position_embeddings": 40960, "eos_token_id": 151645,
    }
    cfg.update(overrides)
    return cfg


def write_safetensors(path: Path, tensors: dict[str, np.ndarray], dtype: str = "BF16",
                      header_patch=None) -> None:
    header, payload, off = {}, [], 0
    for name, bits in tensors.items():
        raw = np.ascontiguousarray(bits, dtype=np.uint16).tobytes()
        header[name] = {"dtype": dtype, "shape": list(bits.shape), "data_offsets": [off, off + len(raw)]}
        payload.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "pt"}
    if header_patch:
        header_patch(header)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in payload:
            f.write(raw)


def write_checkpoint(model_dir: Path, shape: Qwen3Shape, weights: dict[str, np.ndarray], shards: int = 1,
                     config: dict | None = None, header_patch=None, index_patch=None) -> Path:
    model_dir = Path(model_dir)
    model_dir.mkdir(parents=True, exist_ok=True)
    (model_dir / "config.json").write_text(json.dumps(config if config is not None else config_dict(shape)))
    names = list(weights)
    if shards == 1:
        write_safetensors(model_dir / "model.safetensors", weights, header_patch=header_patch)
        return model_dir
    groups = [names[i::shards] for i in range(shards)]
    weight_map, total = {}, 0
    for k, group in enumerate(groups):
        fname = f"model-{k + 1:05d}-of-{shards:05d}.safetensors"
        write_safetensors(model_dir / fname, {n: weights[n] for n in group},
                          header_patch=header_patch if k == 0 else None)
        for n in group:
            weight_map[n] = fname
            total += weights[n].size * 2
    index = {"metadata": {"total_size": total}, "weight_map": weight_map}
    if index_patch:
        index_patch(index)
    (model_dir / "model.safetensors.index.json").write_text(json.dumps(index))
    return model_dir
