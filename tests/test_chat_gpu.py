"""The chat frontend end to end on the GPU: a synthetic checkpoint plus a
word-level tokenizer with a chat template in one model directory, the
frontend run as a program over this package's `qwen3` engine, and its text
compared with the engine's own greedy tokens for the templated prompt."""

import subprocess
import sys

import pytest

from oracle.qwen3_ref import seeded_weights
from tests._ckpt import write_checkpoint
from tests._tokenizer import write_tokenizer
from xpu_playground_b200 import chat
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu


def test_chat_generates_the_engines_tokens(tmp_path):
    from transformers import AutoTokenizer
    shape = PRESETS["tiny-tied"]
    d = write_checkpoint(tmp_path / "m", shape, seeded_weights(shape, 23), shards=1)
    write_tokenizer(d, shape.vocab - 8)  # 8 role/marker tokens after the words: vocab ids exactly
    r = subprocess.run([sys.executable, "-m", "xpu_playground_b200.chat", "--model-dir", str(d),
                        "--prompt", "w11 w12 w13 w14", "--system", "w3 w4", "--max-new-tokens", "24",
                        "--max-seq-len", "64"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    tok = AutoTokenizer.from_pretrained(d, local_files_only=True)
    ids = chat.prompt_ids(tok, "w11 w12 w13 w14", "w3 w4", False)
    with Qwen3Engine(shape, 64) as e:
        e.load_checkpoint(d)
        expected = e.generate(ids, 24, stop_at_eos=True)
    assert len(expected) == 24
    assert r.stdout == tok.decode(expected, skip_special_tokens=False)
