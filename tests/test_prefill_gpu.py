"""Chunked prefill (16 prompt positions per batched tcgen05 step, causal
attention inside each chunk) against the CPU oracles: the batch-1 engine
continued from a chunked prefill must meet the same gates as one fed the
prompt token by token.

* the C restatement of the transformers forward: a 50-token prompt (three
  full chunks and a partial one), the last prompt position's logits and the
  following decode steps within the logit gate;
* qwen3/reference.py's model (transformers golden fixtures): the golden
  token stream's first `prefix` positions prefilled, the remaining positions
  decoded teacher-forced under the fixture gates.
"""

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc
from oracle.qwen3_ref import CDecoder, prompt_ids, seeded_weights
from tests.test_engine_gpu import (FULL_MAXABS, FULL_MEANABS, TOP_MAXABS, logit_gate, near_tie)
from xpu_playground_b200 import _lib
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
f = orc.bf16_to_float


@pytest.mark.parametrize("preset", ["tiny", "tiny-tied"])
def test_prefill_matches_c_oracle(preset):
    shape = PRESETS[preset]
    seed, n, steps = 4321, 50, 64
    ref = CDecoder(shape, seeded_weights(shape, seed), steps)
    eng = Qwen3Engine(shape, steps)
    eng.init_synthetic(seed)
    prompt = prompt_ids(n, shape.vocab, 7)
    for pos in range(n):
        nref, lref = ref.step(prompt[pos], pos)
    nxt = eng.prefill(prompt)
    bad, worst = logit_gate(eng.batch_logits((n - 1) % 16), lref)
    assert bad == 0, f"last prompt position: {bad} logits off, max-abs {worst}"
    assert nxt == nref or near_tie(lref, nxt, nref)
    tok, pos, err = eng.state()
    assert (tok, pos, err) == (nxt, n, 0)
    token, flips = nref, 0
    for pos in range(n, steps):
        nref, lref = ref.step(token, pos)
        got = eng.decode(token, pos)
        bad, worst = logit_gate(eng.logits(), lref)
        assert bad == 0, f"step {pos}: {bad} logits off, max-abs {worst}"
        if got != nref:
            assert near_tie(lref, got, nref)
            flips += 1
        token = nref
    assert flips <= 1
    eng.close()


@pytest.mark.parametrize("fixture,prefix", [("hf_tiny.npz", 20), ("hf_tiny-tied.npz", 29),
                                            ("hf_qwen3-0p6b.npz", 128), ("hf_qwen3-8b-l2.npz", 16)])
def test_prefill_then_decode_matches_transformers(fixture, prefix):
    path = GOLDEN / fixture
    if not path.exists():
        pytest.skip(f"{fixture} not generated")
    fx = np.load(path)
    shape = PRESETS[str(fx["preset"])]
    steps = int(fx["steps"])
    prompt = [int(t) for t in fx["prompt"]]
    ids = [int(t) for t in fx["greedy"]]
    inputs = [prompt[p] if p < len(prompt) else ids[p - 1] for p in range(steps)]
    full = {int(s): i for i, s in enumerate(fx["full_steps"])} if "full_steps" in fx else None
    eng = Qwen3Engine(shape, steps)
    eng.init_synthetic(int(fx["weight_seed"]))
    flips = 0

    def check(pos, nxt, lg):
        nonlocal flips
        if full is None:
            ref_bits = fx["logits"][pos]
            bad, worst = logit_gate(lg, ref_bits)
            assert bad == 0, f"position {pos}: {bad} logits off, max-abs {worst}"
            if nxt != ids[pos]:
                assert near_tie(ref_bits, nxt, ids[pos]), f"position {pos}: {nxt} vs {ids[pos]}"
                flips += 1
        else:
            idx = fx["top_idx"][pos]
            ref_top = f(fx["top_bits"][pos]).astype(np.float64)
            top_dev = np.abs(f(lg[idx]) - ref_top).max()
            assert top_dev <= TOP_MAXABS, f"position {pos}: top-64 max-abs {top_dev}"
            if pos in full:
                d = np.abs(f(lg).astype(np.float64) - f(fx["logits"][full[pos]]))
                assert d.max() <= FULL_MAXABS and d.mean() <= FULL_MEANABS, \
                    f"position {pos}: full max-abs {d.max()}, mean-abs {d.mean()}"
            if nxt != ids[pos]:
                where = np.nonzero(idx == nxt)[0]
                assert where.size and ref_top[0] - ref_top[where[0]] <= TOP_MAXABS, f"position {pos}"
                flips += 1

    nxt = eng.prefill(inputs[:prefix])
    check(prefix - 1, nxt, eng.batch_logits((prefix - 1) % 16))
    for pos in range(prefix, steps):
        nxt = eng.decode(inputs[pos], pos)
        check(pos, nxt, eng.logits())
    assert flips <= max(3, steps // 16)
    eng.close()


def test_prefill_then_device_generation():
    """generate-style continuation: prefill, then device-resident steps from
    the returned token equal host-driven decode from the same state."""
    shape = PRESETS["tiny"]
    prompt = prompt_ids(37, shape.vocab, 11)
    a = Qwen3Engine(shape, 64)
    a.init_synthetic(3)
    t = a.prefill(prompt)
    a.enqueue_steps(5)
    a.synchronize()
    tok_a, pos_a, err = a.state()
    assert err == 0 and pos_a == len(prompt) + 5
    b = Qwen3Engine(shape, 64)
    b.init_synthetic(3)
    assert b.prefill(prompt) == t
    for i in range(5):
        t = b.decode(t, len(prompt) + i)
    assert t == tok_a
    with pytest.raises(_lib.XpuError, match="maximum sequence"):
        b.prefill([1] * 65)
    a.close(); b.close()
