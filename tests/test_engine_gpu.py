"""Qwen3 decode engine on the GPU against the CPU oracles.

* the device generators reproduce the oracle's seeded data bit for bit;
* per step, teacher-forced on the same tokens: logits within 2e-2 max-abs of
  the C restatement of the transformers forward and of qwen3/reference.py's
  model itself (golden fixtures), greedy ids equal except bf16 near-ties;
* device-resident generation equals step-by-step decoding bit for bit;
* host-side argument checks of the engine API.
"""

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from oracle.qwen3_ref import CDecoder, prompt_ids, seeded_weights
from tests._util import to_bits
from xpu_playground_b200 import _lib
from xpu_playground_b200.qwen3 import Qwen3Engine
from xpu_playground_b200.qwen3_config import PRESETS

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
f = orc.bf16_to_float
LOGIT_TOL = 2e-2  # north-star: Qwen3 logits within 2e-2 max-abs


def logit_gate(actual_bits, ref_bits):
    """Per logit: |a - e| <= max(2e-2, two bf16 steps at |e|).

    2e-2 max-abs is the north-star gate. Logits of the 28/36-layer models
    reach |e| ~ 3, where one bf16 step is 2^-6 = 0.0156; two correct FP32-
    accumulating implementations of the same bf16 model then differ by up to
    two steps (0.031): the C restatement of the transformers forward differs
    from transformers itself by exactly that on the 0.6B fixture, while
    transformers is bit-stable across thread counts. Below |e| = 2 the gate
    is the plain 2e-2."""
    a, e = f(actual_bits).astype(np.float64), f(ref_bits).astype(np.float64)
    step = np.exp2(np.floor(np.log2(np.maximum(np.abs(e), 1e-30))) - 7)
    bad = np.abs(a - e) > np.maximum(LOGIT_TOL, 2 * step)
    return int(bad.sum()), float(np.abs(a - e).max())


def near_tie(ref_bits, a, b_):
    lv = f(ref_bits)
    gap = abs(float(lv[a]) - float(lv[b_]))
    return gap <= 2 * 2.0 ** (math.floor(math.log2(max(abs(float(lv[a])), 1e-30))) - 7)


@pytest.mark.parametrize("n", [1, 1000, 65537])
def test_device_generators_match_oracle(n):
    L = _lib.load()
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    _lib.check(L.xpu_fill_normal_bf16(out.data_ptr(), n, 77, 5, 0.02, None))
    assert np.array_equal(to_bits(out), orc.normal_bf16(n, 77, 5, 0.02))
    for dtype, fp16 in ((_lib.XPU_BF16, False), (_lib.XPU_FP16, True)):
        _lib.check(L.xpu_fill_uniform16(dtype, out.data_ptr(), n, 9, 3, None))
        assert np.array_equal(to_bits(out), orc.uniform16(n, 9, 3, fp16))


@pytest.mark.parametrize("preset", ["tiny", "tiny-tied"])
def test_engine_matches_c_oracle(preset):
    shape = PRESETS[preset]
    seed, steps = 4321, 40
    weights = seeded_weights(shape, seed)
    ref = CDecoder(shape, weights, steps)
    eng = Qwen3Engine(shape, steps)
    eng.init_synthetic(seed)
    prompt = prompt_ids(6, shape.vocab, 1)
    token, flips = prompt[0], 0
    for pos in range(steps):
        t = prompt[pos] if pos < len(prompt) else token
        nxt_ref, lref = ref.step(t, pos)
        nxt = eng.decode(t, pos)
        lg = eng.logits()
        bad, worst = logit_gate(lg, lref)
        assert bad == 0, f"step {pos}: {bad} logits off, max-abs {worst}"
        if nxt != nxt_ref:
            assert near_tie(lref, nxt, nxt_ref), f"step {pos}: {nxt} vs {nxt_ref}"
            flips += 1
        token = nxt_ref
    assert flips <= 1
    # No bit-level bound: one last-place difference in a large residual
    # element moves the final RMSNorm scale and with it many logits by one
    # bf16 step (the C oracle and transformers differ from each other the
    # same way), so the tolerance above is the gate.
    eng.close()


def test_set_tensor_equals_init_synthetic():
    shape = PRESETS["tiny-tied"]
    a = Qwen3Engine(shape, 16)
    a.init_synthetic(99)
    b = Qwen3Engine(shape, 16)
    b.load_weights(seeded_weights(shape, 99))
    for pos, tok in enumerate([5, 17, 3000, 2, 9]):
        assert a.decode(tok, pos) == b.decode(tok, pos)
        assert np.array_equal(a.logits(), b.logits())
    a.close(); b.close()


# Gates for the 151936-vocabulary fixtures (28-layer 0.6B, 8B shapes). The
# C restatement of the transformers forward (same rounding points, FP32
# accumulation in another order) differs from transformers itself on the
# 0.6B fixture by full-logit max-abs 0.055 and mean-abs 0.0098, top-64
# max-abs 0.047: the noise floor between two correct implementations of a
# deep bf16 model. The engine measures 0.0547 / 0.0094 / 0.047 against the
# fixture on B200 (and 0.059 / 0.0095 / 0.047 against the C restatement
# over 256 steps): it is held to the floor plus ~10%.
FULL_MAXABS, FULL_MEANABS, TOP_MAXABS = 0.06, 0.0105, 0.052

# Paths whose projections accumulate on the tensor cores (TMEM: the batched
# step's GEMMs, the dense prefill) carry more FP32 rounding than the decode
# GEMVs' FMA chains: against the C restatement on the 8B shapes the dense
# prefill's distance is 1.33x the decode path's in max-abs, 1.21x in
# mean-abs and 1.17x in relative L2 (tests/test_prefill_dense_gpu.py). Their
# gates are the ones above scaled by TC_SCALE.
TC_SCALE = 1.25


@pytest.mark.parametrize("fixture", ["hf_tiny.npz", "hf_tiny-tied.npz", "hf_qwen3-0p6b.npz",
                                     "hf_qwen3-8b-l2.npz"])
def test_engine_matches_transformers_fixture(fixture):
    """qwen3/reference.py's model (transformers, bf16 eager) on the same
    seeded checkpoint, teacher-forced on its own greedy path."""
    path = GOLDEN / fixture
    if not path.exists():
        pytest.skip(f"{fixture} not generated")
    fx = np.load(path)
    shape = PRESETS[str(fx["preset"])]
    steps = int(fx["steps"])
    eng = Qwen3Engine(shape, steps)
    eng.init_synthetic(int(fx["weight_seed"]))
    prompt = [int(t) for t in fx["prompt"]]
    ids = [int(t) for t in fx["greedy"]]
    full = {int(s): i for i, s in enumerate(fx["full_steps"])} if "full_steps" in fx else None
    flips = 0
    for pos in range(steps):
        t = prompt[pos] if pos < len(prompt) else ids[pos - 1]
        nxt = eng.decode(t, pos)
        lg = eng.logits()
        if full is None:
            ref_bits = fx["logits"][pos]
            bad, worst = logit_gate(lg, ref_bits)
            assert bad == 0, f"step {pos}: {bad} logits off, max-abs {worst}"
            if nxt != ids[pos]:
                assert near_tie(ref_bits, nxt, ids[pos]), f"step {pos}: {nxt} vs {ids[pos]}"
                flips += 1
        else:
            idx = fx["top_idx"][pos]
            ref_top = f(fx["top_bits"][pos]).astype(np.float64)
            top_dev = np.abs(f(lg[idx]) - ref_top).max()
            assert top_dev <= TOP_MAXABS, f"step {pos}: top-64 max-abs {top_dev}"
            if pos in full:
                d = np.abs(f(lg).astype(np.float64) - f(fx["logits"][full[pos]]))
                assert d.max() <= FULL_MAXABS and d.mean() <= FULL_MEANABS, \
                    f"step {pos}: full max-abs {d.max()}, mean-abs {d.mean()}"
            if nxt != ids[pos]:
                where = np.nonzero(idx == nxt)[0]
                assert where.size, f"step {pos}: {nxt} not in the reference's top 64"
                gap = ref_top[0] - ref_top[where[0]]
                assert gap <= TOP_MAXABS, f"step {pos}: {nxt} vs {ids[pos]}, reference gap {gap}"
                flips += 1
    assert flips <= max(1, steps // 32)
    eng.close()


def test_generate_equals_stepwise_decode():
    shape = PRESETS["tiny"]
    prompt = prompt_ids(10, shape.vocab, 3)
    eng = Qwen3Engine(shape, 64)
    eng.init_synthetic(5)
    gen = eng.generate(prompt, 30)
    eng2 = Qwen3Engine(shape, 64)
    eng2.init_synthetic(5)
    tok = None
    for pos in range(len(prompt)):
        tok = eng2.decode(prompt[pos], pos)
    steps = [tok]
    for i in range(29):
        steps.append(eng2.decode(steps[-1], len(prompt) + i))
    assert gen == steps
    # device-resident enqueue from a set state continues the same sequence
    eng.set_state(steps[-1], len(prompt) + 29)
    eng.enqueue_steps(1)
    eng.synchronize()
    nxt, pos, err = eng.state()
    assert err == 0 and pos == len(prompt) + 30
    assert nxt == eng2.decode(steps[-1], len(prompt) + 29)
    eng.close(); eng2.close()


def test_engine_argument_errors():
    shape = PRESETS["tiny"]
    eng = Qwen3Engine(shape, 8)
    with pytest.raises(_lib.XpuError, match="no weights"):
        eng.decode(1, 0)
    eng.init_synthetic(1)
    with pytest.raises(_lib.XpuError, match="maximum sequence"):
        eng.decode(1, 8)
    with pytest.raises(_lib.XpuError, match="vocabulary"):
        eng.decode(shape.vocab, 0)
    with pytest.raises(_lib.XpuError, match="elements"):
        eng.set_tensor("model.norm.weight", np.zeros(3, np.uint16))
    with pytest.raises(_lib.XpuError, match="unknown"):
        eng.set_tensor("model.layers.0.bogus", np.zeros(3, np.uint16))
    with pytest.raises(_lib.XpuError):
        Qwen3Engine(PRESETS["tiny"], 0)
    eng.close()


@pytest.mark.parametrize("preset", ["tiny", "tiny-tied", "qwen3-8b-l2"])
def test_persistent_step_equals_graph_step(preset):
    """The single-kernel persistent step and the multi-kernel CUDA-graph step
    run the same per-item math: logits and tokens must agree bit for bit."""
    shape = PRESETS[preset]
    steps = 12
    a = Qwen3Engine(shape, 160, mode="persistent")
    b = Qwen3Engine(shape, 160, mode="graph")
    a.init_synthetic(31)
    b.init_synthetic(31)
    prompt = prompt_ids(5, shape.vocab, 2)
    ta = tb = None
    for pos in range(steps):
        t = prompt[pos] if pos < len(prompt) else ta
        ta, tb = a.decode(t, pos), b.decode(t, pos)
        assert ta == tb, f"step {pos}"
        assert np.array_equal(a.logits(), b.logits()), f"step {pos}"
    # long context: jump to position 140 (chunks 0..1 of attention)
    assert a.decode(7, 140) == b.decode(7, 140)
    assert np.array_equal(a.logits(), b.logits())
    a.close(); b.close()


@pytest.mark.parametrize("prompt_len", [18930, 37880])
def test_persistent_step_equals_graph_step_at_long_contexts(prompt_len):
    """Contexts whose 128-position chunks outnumber the SMs: the persistent
    step gives each CTA runs of 2 (above 148 chunks) or 3 (above 296 chunks)
    chunks of a kv head per attention item, the graph step one chunk per CTA.
    Generation crosses those boundaries (148 -> 149 and 296 -> 297 chunks)
    with identical tokens and identical final logits."""
    shape = PRESETS["tiny"]
    prompt = prompt_ids(prompt_len, shape.vocab, 11)
    out = []
    for mode in ("persistent", "graph"):
        with Qwen3Engine(shape, 40960, mode=mode) as e:
            e.init_synthetic(13)
            out.append((e.generate(prompt, 24), e.logits()))
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][1], out[1][1])
