"""Parity at the benchmarked depth: the engine against the C restatement of
the transformers forward (oracle/xpu_oracle.c) on the full 36-layer
Qwen3-8B shape and, free-running, on the 28-layer Qwen3-0.6B shape.

What two correct implementations of these models can agree on: the C
restatement and transformers itself (qwen3/reference.py's model, bf16
eager), same weights and tokens, differ at 36 layers by full-logit max-abs
0.20-0.25 and relative L2 3.4-4.4% per step (logits up to |5.9|, measured
on one B200 box's host for 12 steps; greedy ids equal except two exact
ties), because FP32 accumulation order decides which bf16 roundings land
one step apart and 36 layers carry those differences on. The engine is held
to that noise floor with a 1.5x margin, to bit-identity between its two
decode paths at full depth, and to identical greedy tokens except where the
reference's own top two are within two bf16 steps (a tie for any
implementation).
"""

import math

import numpy as np
import pytest

from oracle import oracle as orc
from oracle.qwen3_ref import CDecoder, prompt_ids, seeded_weights
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu
f = orc.bf16_to_float

# C restatement vs transformers at 36 layers: worst per-step max-abs 0.245,
# relative L2 0.044 (module docstring); 1.5x of it.
DEEP_MAXABS, DEEP_REL_L2 = 0.37, 0.066


def near_tie(ref_bits, a, b) -> bool:
    """The reference's logits of tokens a and b are within two bf16 steps."""
    lv = f(ref_bits).astype(np.float64)
    gap = abs(lv[a] - lv[b])
    return gap <= 2 * 2.0 ** (math.floor(math.log2(max(abs(lv[a]), abs(lv[b]), 1e-30))) - 7)


def test_qwen3_8b_full_depth_against_c_oracle_and_graph_path():
    shape = PRESETS["qwen3-8b"]
    seed, plen, steps = 8, 8, 12
    weights = seeded_weights(shape, seed)
    ref = CDecoder(shape, weights, 32)
    del weights
    pers = Qwen3Engine(shape, 32, mode="persistent")
    graph = Qwen3Engine(shape, 32, mode="graph")
    pers.init_synthetic(seed)
    graph.init_synthetic(seed)
    prompt = prompt_ids(plen, shape.vocab, 5)
    tok, flips = None, 0
    for pos in range(plen + steps):
        t = prompt[pos] if pos < plen else tok  # teacher-forced on the reference's greedy path
        nref, lref = ref.step(t, pos)
        n, ng = pers.decode(t, pos), graph.decode(t, pos)
        lg = pers.logits()
        assert n == ng and np.array_equal(lg, graph.logits()), f"step {pos}: decode paths differ"
        e, a = f(lref).astype(np.float64), f(lg).astype(np.float64)
        maxabs, rel = np.abs(a - e).max(), np.linalg.norm(a - e) / np.linalg.norm(e)
        assert maxabs <= DEEP_MAXABS and rel <= DEEP_REL_L2, f"step {pos}: max-abs {maxabs}, rel-L2 {rel}"
        if n != nref:
            assert near_tie(lref, n, nref), f"step {pos}: {n} vs {nref}"
            flips += 1
        tok = nref
    assert flips <= 2
    pers.close()
    graph.close()


def test_qwen3_0p6b_free_running_greedy_against_c_oracle():
    """a 128-token prompt, then 128 greedy tokens, each
    implementation feeding back its own tokens. The sequences must agree
    until the reference meets a near-tie; past a divergence the inputs
    differ, so nothing further is compared."""
    shape = PRESETS["qwen3-0.6b"]
    seed, plen, n_new = 2026, 128, 128
    ref = CDecoder(shape, seeded_weights(shape, seed), plen + n_new)
    prompt = prompt_ids(plen, shape.vocab, 3)
    with Qwen3Engine(shape, plen + n_new) as eng:
        eng.init_synthetic(seed)
        got = eng.generate(prompt, n_new)
    want, tok, last_bits = [], None, []
    for pos in range(plen + n_new - 1):
        tok, bits = ref.step(prompt[pos] if pos < plen else tok, pos)
        if pos >= plen - 1:
            want.append(tok)
            last_bits.append(bits)
    same = next((i for i in range(n_new) if got[i] != want[i]), n_new)
    if same < n_new:
        assert near_tie(last_bits[same], got[same], want[same]), \
            f"generated token {same} differs ({got[same]} vs {want[same]}) without a near-tie"
    # the measured span on one B200: the first 26 tokens agree, then the
    # reference meets an exact tie (both logits 0 apart in bf16)
    assert same >= 16, f"only {same} identical greedy tokens"
