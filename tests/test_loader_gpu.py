"""Checkpoint loading on the GPU: a safetensors checkpoint written from the
seeded weights decodes to bit-identical logits as the same weights generated
on the device, for sharded and single-file, tied and untied checkpoints."""

import numpy as np
import pytest

from oracle.qwen3_ref import prompt_ids, seeded_weights
from tests._ckpt import write_checkpoint
from xpu_playground_b200._lib import XpuError
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("preset,shards", [("tiny", 3), ("tiny-tied", 1), ("qwen3-0.6b", 2)])
def test_loaded_checkpoint_matches_device_weights(tmp_path, preset, shards):
    shape = PRESETS[preset]
    seed = 17
    d = write_checkpoint(tmp_path / preset, shape, seeded_weights(shape, seed), shards=shards)
    prompt = prompt_ids(8, shape.vocab, seed=2)
    with Qwen3Engine(shape, 64) as a, Qwen3Engine(shape, 64) as b:
        a.load_checkpoint(d)
        b.init_synthetic(seed)
        for pos, tok in enumerate(prompt):
            assert a.decode(tok, pos) == b.decode(tok, pos)
            assert np.array_equal(a.logits(), b.logits())


def test_load_rejects_a_checkpoint_of_another_shape(tmp_path):
    d = write_checkpoint(tmp_path / "tiny", PRESETS["tiny"], seeded_weights(PRESETS["tiny"], 1))
    with Qwen3Engine(PRESETS["tiny-tied"], 16) as e:
        with pytest.raises(XpuError, match="checkpoint config does not match the engine"):
            e.load_checkpoint(d)


def test_qwen3_cli_generates_like_the_engine(tmp_path):
    """The qwen3 program (reference main.cpp's flags and JSON output) on a
    checkpoint directory gives the engine's greedy tokens."""
    import json
    import subprocess
    from xpu_playground_b200 import build
    shape = PRESETS["tiny-tied"]
    d = write_checkpoint(tmp_path / "m", shape, seeded_weights(shape, 5), shards=2)
    prompt = prompt_ids(12, shape.vocab, seed=9)
    (tmp_path / "ids.txt").write_text(" ".join(map(str, prompt)) + "\n")
    r = subprocess.run([str(build.BIN_DIR / "qwen3"), "--model-dir", str(d), "--input-ids", str(tmp_path / "ids.txt"),
                        "--max-new-tokens", "20", "--max-seq-len", "64"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    with Qwen3Engine(shape, 64) as e:
        e.load_checkpoint(d)
        assert out["generated_ids"] == e.generate(prompt, 20, stop_at_eos=True)
