"""Checkpoint reading on CPU: config.json and safetensors validation with
the reference loader's rules (qwen3/model.cpp:376-495), generalised to any
Qwen3 shape with head_dim 128, tied embeddings and single-file checkpoints."""

import json

import numpy as np
import pytest

from oracle.qwen3_ref import seeded_weights
from tests._ckpt import config_dict, write_checkpoint, write_safetensors
from xpu_playground_b200._lib import XpuError
from xpu_playground_b200.qwen3 import read_config, validate_checkpoint
from xpu_playground_b200.qwen3_config import PRESETS

TINY, TIED = PRESETS["tiny"], PRESETS["tiny-tied"]


@pytest.fixture(scope="module")
def tiny_weights():
    return seeded_weights(TINY, 3)


@pytest.fixture(scope="module")
def tied_weights():
    return seeded_weights(TIED, 4)


def expect_error(model_dir, needle):
    with pytest.raises(XpuError) as e:
        validate_checkpoint(model_dir)
    assert needle in str(e.value), str(e.value)


@pytest.mark.parametrize("shards", [1, 3])
def test_valid_checkpoints(tmp_path, tiny_weights, shards):
    d = write_checkpoint(tmp_path / "m", TINY, tiny_weights, shards=shards)
    shape, nbytes = validate_checkpoint(d)
    assert shape == TINY
    assert nbytes == sum(w.size * 2 for w in tiny_weights.values())
    assert read_config(d) == TINY


def test_tied_checkpoint_has_no_lm_head(tmp_path, tied_weights):
    d = write_checkpoint(tmp_path / "m", TIED, tied_weights)
    assert validate_checkpoint(d)[0] == TIED
    bad = dict(tied_weights, **{"lm_head.weight": tied_weights["model.embed_tokens.weight"]})
    expect_error(write_checkpoint(tmp_path / "m2", TIED, bad), "unexpected tensor in checkpoint: lm_head.weight")


def test_real_shapes_config_only(tmp_path):
    for name in ("qwen3-0.6b", "qwen3-8b"):
        d = tmp_path / name
        d.mkdir()
        (d / "config.json").write_text(json.dumps(config_dict(PRESETS[name])))
        assert read_config(d) == PRESETS[name]


@pytest.mark.parametrize("override,needle", [
    ({"model_type": "llama"}, "model_type must be \"qwen3\""),
    ({"hidden_act": "gelu"}, "hidden_act must be \"silu\""),
    ({"torch_dtype": "float16"}, "weights must be bfloat16"),
    ({"head_dim": 64}, "head_dim must be 128"),
    ({"rope_scaling": {"type": "yarn", "factor": 4.0}}, "rope_scaling is not supported"),
    ({"num_key_value_heads": 3}, "multiple of num_key_value_heads"),
    ({"hidden_size": -1}, "'hidden_size' must be an unsigned 32-bit integer"),
    ({"tie_word_embeddings": "no"}, "'tie_word_embeddings' must be true or false"),
])
def test_config_rejections(tmp_path, tiny_weights, override, needle):
    d = write_checkpoint(tmp_path / "m", TINY, tiny_weights, config=config_dict(TINY, **override))
    expect_error(d, needle)


def test_config_missing_field_and_bad_json(tmp_path, tiny_weights):
    cfg = config_dict(TINY)
    del cfg["rope_theta"]
    expect_error(write_checkpoint(tmp_path / "a", TINY, tiny_weights, config=cfg), "missing field 'rope_theta'")
    d = write_checkpoint(tmp_path / "b", TINY, tiny_weights)
    (d / "config.json").write_text('{"hidden_size": 256,')
    expect_error(d, "malformed JSON")
    # transformers 5 writes "dtype" instead of "torch_dtype"
    cfg = config_dict(TINY)
    cfg["dtype"] = cfg.pop("torch_dtype")
    assert validate_checkpoint(write_checkpoint(tmp_path / "c", TINY, tiny_weights, config=cfg))[0] == TINY


def test_tensor_rejections(tmp_path, tiny_weights):
    w = dict(tiny_weights)
    missing = {k: v for k, v in w.items() if k != "model.layers.1.mlp.up_proj.weight"}
    expect_error(write_checkpoint(tmp_path / "a", TINY, missing),
                 "missing tensor: model.layers.1.mlp.up_proj.weight")
    extra = dict(w, **{"model.layers.9.mlp.up_proj.weight": w["model.layers.1.mlp.up_proj.weight"]})
    expect_error(write_checkpoint(tmp_path / "b", TINY, extra), "unexpected tensor in checkpoint")
    wrong = dict(w, **{"model.layers.0.self_attn.o_proj.weight": np.zeros((256, 256), np.uint16)})
    expect_error(write_checkpoint(tmp_path / "c", TINY, wrong), "wrong shape for tensor model.layers.0.self_attn.o_proj")

    def f32(h):
        h["model.norm.weight"]["dtype"] = "F32"
    expect_error(write_checkpoint(tmp_path / "d", TINY, w, header_patch=f32), "dtype F32; BF16 is required")

    def overlap(h):
        h["model.norm.weight"]["data_offsets"] = list(h["model.embed_tokens.weight"]["data_offsets"][:1]) * 2
        h["model.norm.weight"]["data_offsets"][1] += 512
    expect_error(write_checkpoint(tmp_path / "e", TINY, w, header_patch=overlap), "overlapping tensor payloads")

    def beyond(h):
        h["model.norm.weight"]["data_offsets"] = [10**9, 10**9 + 512]
    expect_error(write_checkpoint(tmp_path / "f", TINY, w, header_patch=beyond), "extends beyond")

    def size(h):
        h["model.norm.weight"]["shape"] = [128]
    expect_error(write_checkpoint(tmp_path / "g", TINY, w, header_patch=size), "byte size does not match")


def test_index_rejections(tmp_path, tiny_weights):
    def total(i):
        i["metadata"]["total_size"] += 2
    expect_error(write_checkpoint(tmp_path / "a", TINY, tiny_weights, shards=2, index_patch=total),
                 "does not match the tensor payloads")

    def escape(i):
        i["weight_map"]["model.norm.weight"] = "../x.safetensors"
    expect_error(write_checkpoint(tmp_path / "b", TINY, tiny_weights, shards=2, index_patch=escape),
                 "invalid shard name")
    d = write_checkpoint(tmp_path / "c", TINY, tiny_weights, shards=2)
    # a shard holding a tensor the index assigns elsewhere
    first = sorted(d.glob("model-00001-*.safetensors"))[0]
    idx = json.loads((d / "model.safetensors.index.json").read_text())
    moved = next(n for n, f in idx["weight_map"].items() if f != first.name)
    idx["weight_map"][moved] = first.name
    (d / "model.safetensors.index.json").write_text(json.dumps(idx))
    expect_error(d, "does not hold")
    empty = tmp_path / "empty"
    empty.mkdir()
    (empty / "config.json").write_text(json.dumps(config_dict(TINY)))
    expect_error(empty, "neither model.safetensors.index.json nor model.safetensors found")


def test_truncated_header(tmp_path, tiny_weights):
    d = write_checkpoint(tmp_path / "m", TINY, tiny_weights)
    raw = (d / "model.safetensors").read_bytes()
    (d / "model.safetensors").write_bytes(raw[:20])
    expect_error(d, "invalid safetensors header length")
