"""Dense prefill (xpu_qwen3_prefill_dense: every prompt position through
each layer together, tcgen05 GEMMs against the stored weights, causal
attention over the cache) against the CPU oracles:

* the C restatement of the transformers forward: the last prompt position's
  logits (a 50-token prompt, one of 2100 tokens that takes two segments, and
  the 8B layer shapes) and the decode steps that follow, under logit_gate;
* qwen3/reference.py's model (transformers golden fixtures): the golden
  token stream's first `prefix` positions prefilled densely, the remaining
  positions decoded teacher-forced under the fixture gates, with the
  per-logit two-bf16-step rule of logit_gate applied to the top-64 and
  full-logit checks (top_gate).
"""

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc
from oracle.qwen3_ref import CDecoder, prompt_ids, seeded_weights
from tests.test_engine_gpu import (FULL_MEANABS, TOP_MAXABS, logit_gate, near_tie)
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
f = orc.bf16_to_float


def top_gate(ref_top):
    """Per top-64 logit: TOP_MAXABS, or two bf16 steps of the reference value
    where that is larger - logit_gate's rule for two correct FP32-
    accumulating implementations. The dense GEMMs sum in another order than
    the decode GEMVs, so K/V entries land a rounding apart; on the 8B-shaped
    fixture a logit of 6.0 then moves by two steps (0.0625), above the
    absolute 0.052 that the decode-only path stays under."""
    step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref_top), 1e-30))) - 7)
    return np.maximum(TOP_MAXABS, 2 * step)


@pytest.mark.parametrize("preset,n,steps", [("tiny", 50, 64), ("tiny-tied", 50, 64), ("tiny", 2100, 2110),
                                            ("qwen3-8b-l2", 16, 32)])
def test_dense_prefill_matches_c_oracle(preset, n, steps):
    shape = PRESETS[preset]
    seed = 4321
    ref = CDecoder(shape, seeded_weights(shape, seed), steps)
    prompt = prompt_ids(n, shape.vocab, 7)
    for pos in range(n):
        nref, lref = ref.step(prompt[pos], pos, want_logits=pos == n - 1)
    with Qwen3Engine(shape, steps) as eng:
        eng.init_synthetic(seed)
        nxt = eng.prefill_dense(prompt)
        bad, worst = logit_gate(eng.logits(), lref)
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


@pytest.mark.parametrize("fixture,prefix", [("hf_tiny.npz", 20), ("hf_tiny-tied.npz", 29),
                                            ("hf_qwen3-0p6b.npz", 128), ("hf_qwen3-8b-l2.npz", 16)])
def test_dense_prefill_then_decode_matches_transformers(fixture, prefix):
    fx = np.load(GOLDEN / fixture)
    shape = PRESETS[str(fx["preset"])]
    steps = int(fx["steps"])
    prompt = [int(t) for t in fx["prompt"]]
    ids = [int(t) for t in fx["greedy"]]
    inputs = [prompt[p] if p < len(prompt) else ids[p - 1] for p in range(steps)]
    full = {int(s): i for i, s in enumerate(fx["full_steps"])} if "full_steps" in fx else None
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
            dev = np.abs(f(lg[idx]) - ref_top)
            assert np.all(dev <= top_gate(ref_top)), f"position {pos}: top-64 max-abs {dev.max()}"
            if pos in full:
                # per logit the full-logit rule of logit_gate (two bf16 steps
                # of the reference value above 2e-2), and the mean-abs gate
                bad, worst = logit_gate(lg, fx["logits"][full[pos]])
                d = np.abs(f(lg).astype(np.float64) - f(fx["logits"][full[pos]]))
                assert bad == 0 and d.mean() <= FULL_MEANABS, \
                    f"position {pos}: {bad} logits off, max-abs {worst}, mean-abs {d.mean()}"
            if nxt != ids[pos]:
                where = np.nonzero(idx == nxt)[0]
                assert where.size and ref_top[0] - ref_top[where[0]] <= TOP_MAXABS, f"position {pos}"
                flips += 1

    with Qwen3Engine(shape, steps) as eng:
        eng.init_synthetic(int(fx["weight_seed"]))
        nxt = eng.prefill_dense(inputs[:prefix])
        check(prefix - 1, nxt, eng.logits())
        for pos in range(prefix, steps):
            nxt = eng.decode(inputs[pos], pos)
            check(pos, nxt, eng.logits())
    assert flips <= max(3, steps // 16)


def test_dense_prefill_then_device_generation():
    """Device-resident steps continue from the dense prefill's state exactly
    as host-driven decode does."""
    shape = PRESETS["tiny"]
    prompt = prompt_ids(97, shape.vocab, 11)
    with Qwen3Engine(shape, 128) as a, Qwen3Engine(shape, 128) as b:
        a.init_synthetic(3)
        b.init_synthetic(3)
        t = a.prefill_dense(prompt)
        a.enqueue_steps(5)
        a.synchronize()
        tok_a, pos_a, err = a.state()
        assert err == 0 and pos_a == len(prompt) + 5
        assert b.prefill_dense(prompt) == t
        for i in range(5):
            t = b.decode(t, len(prompt) + i)
        assert t == tok_a
