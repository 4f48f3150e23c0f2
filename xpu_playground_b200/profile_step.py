"""Profile one Qwen3 decode step (the launch that ncu captures, or a phase trace).

    python -m xpu_playground_b200.profile_step --preset qwen3-8b-l2 --context 2048 --warm 2
    python -m xpu_playground_b200.profile_step --preset qwen3-8b --context 2048 --trace

The default run builds a seeded synthetic model, places the decode state at
`--context` cached positions (the KV cache contents do not change the work),
and runs `--warm` + 1 decode steps, so that the step to capture under
`ncu --clock-control none -k regex:k_step -s <warm> -c 1` is the last one. Weight initialisation
launches one fill kernel per tensor before that.

Under torchrun the ranks run one tensor-parallel engine and rank 0 prints
every rank's report:

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        -m xpu_playground_b200.profile_step --preset qwen3-8b --trace

--trace re-runs with XPU_STEP_TRACE=1 and prints, per phase of the persistent
step, the mean/max over CTAs of the time spent staging the activation,
streaming its items, finishing (arrivals and epilogues) and in the grid
barrier, averaged over layers.

--batch B profiles the batched step (B sequences, one CUDA graph of tcgen05
GEMMs and attention kernels per step) instead: every sequence is prefilled
through the batched step to `--context` positions, `--warm` steps follow, and
one last step runs between cudaProfilerStart/Stop, so the launch list of one
step is

    ncu --metrics gpu__time_duration.sum --clock-control none --profile-from-start off \
        --csv python -m xpu_playground_b200.profile_step --batch 16 --context 512

--prefill N profiles the dense prefill of an N-token prompt instead (one
untimed call, then one between cudaProfilerStart/Stop, whose wall time is
printed), so that its launch list is

    ncu --metrics gpu__time_duration.sum --clock-control none --profile-from-start off \
        --csv python -m xpu_playground_b200.profile_step --prefill 2048

With --trace it prints that step's per-kernel timeline (XPU_BATCH_TRACE=1):
per kernel kind the critical-path time (end minus the previous kernel's end),
when its wait on the previous kernel returned, when its last CTA saw its first
stage and its final accumulator, and the epilogue tail.
"""

from __future__ import annotations

import argparse
import ctypes
import os

import numpy as np

PHASES = ["qkv", "scores", "pv", "o_proj", "gate_up", "down"]
PARTS = ["stage", "items", "finish", "barrier"]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--preset", default="qwen3-8b")
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--warm", type=int, default=2)
    ap.add_argument("--mode", choices=["persistent", "graph"], default="persistent")
    ap.add_argument("--trace", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="profile the batched step of this many sequences")
    ap.add_argument("--prefill", type=int, default=0, help="profile the dense prefill of this many tokens")
    args = ap.parse_args()
    if args.prefill:
        prefill_profile(args)
        return
    if args.batch:
        batch_profile(args)
        return
    if args.trace:
        os.environ["XPU_STEP_TRACE"] = "1"

    from .qwen3 import Qwen3Engine
    from .qwen3_config import PRESETS

    shape = PRESETS[args.preset]
    # Under torchrun (WORLD_SIZE > 1) the ranks run one tensor-parallel
    # engine (one GPU each) and rank 0 reports.
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    eng = Qwen3Engine(shape, args.context + args.warm + 8, device=local, tp_rank=rank, tp_size=world,
                      mode=args.mode if world == 1 else "persistent")
    eng.init_synthetic(1)
    if world > 1:
        eng.connect_tensor_parallel()
    eng.set_state(5, args.context)
    eng.enqueue_steps(args.warm + 1)
    eng.synchronize()
    tok, pos, err = eng.state()
    report = [f"{args.preset}: position {pos}, last token {tok}, error {err}, tp {world}, rank {rank}, "
              f"kernels/step {eng.info().kernels_per_step}, fill launches {len(shape.tensor_names())}"]
    stamps = None
    if args.trace:
        report += trace_table(eng, shape.layers)
        stamps = trace_stamps(eng, shape.layers)
    if world > 1:
        # every rank's table, printed by rank 0 in rank order
        reports = [None] * world
        dist.all_gather_object(reports, report)
        every = [None] * world
        dist.all_gather_object(every, stamps)
        dist.barrier()
        eng.close()
        dist.destroy_process_group()
    else:
        reports, every = [report], [stamps]
        eng.close()
    if rank == 0:
        for r in reports:
            print("\n".join(r))
        if args.trace and world > 1:
            print("\n".join(exchange_skew(every, shape.layers)))


def trace_stamps(eng, L: int) -> np.ndarray:
    """Raw globaltimer stamps of the last step, [cta][event] (ns)."""
    from . import _lib
    n = ctypes.c_uint32()
    _lib.check(eng.lib.xpu_qwen3_trace(eng._h, None, 0, ctypes.byref(n)))
    buf = np.zeros(n.value, np.uint64)
    _lib.check(eng.lib.xpu_qwen3_trace(eng._h, buf.ctypes.data, n.value, ctypes.byref(n)))
    return buf.reshape(-1, 1 + 24 * L + 2).astype(np.int64)


def exchange_skew(every: list, L: int) -> list[str]:
    """Cross-rank view of the two exchanges per layer (globaltimer stamps of
    different GPUs compared directly, so rank clock offsets show up too):
    per exchange, the spread over ranks of the time the rank's last CTA
    finished its partial stores, and how long after the last rank's last
    store each rank's CTAs finished staging (first / last CTA)."""
    out = ["exchange skew (us, mean over layers): stores-done spread over ranks | staging done after the last "
           "rank's last store, first CTA / last CTA per rank"]
    # o_proj: phase 3 items end = event 1+24l+4*3+1; its staging ends at gate_up stage = 1+24l+4*4+0
    # down:   phase 5 items end = 1+24l+4*5+1; staging ends at next qkv stage = 1+24(l+1)+0 (last layer: skip)
    for name, ph, nxt in (("o_proj", 3, lambda l: 1 + 24 * l + 16), ("down", 5, lambda l: 1 + 24 * (l + 1))):
        spread, first_after, last_after = [], [], []
        for l in range(L - 1):
            e_items = 1 + 24 * l + 4 * ph + 1
            done = np.array([t[:, e_items].max() for t in every])
            ready_first = np.array([t[:, nxt(l)].min() for t in every])
            ready_last = np.array([t[:, nxt(l)].max() for t in every])
            spread.append(done.max() - done.min())
            first_after.append(ready_first - done.max())
            last_after.append(ready_last - done.max())
        fa, la = np.mean(first_after, axis=0) / 1e3, np.mean(last_after, axis=0) / 1e3
        out.append(f"{name:7s} spread {np.mean(spread) / 1e3:6.2f} | " +
                   "  ".join(f"r{r} {fa[r]:5.2f}/{la[r]:5.2f}" for r in range(len(every))))
    return out


def trace_table(eng, L: int) -> list[str]:
    """Per phase of the last persistent step: mean/max over CTAs (averaged
    over layers) of staging, items, finishing and barrier time."""
    from . import _lib
    n = ctypes.c_uint32()
    _lib.check(eng.lib.xpu_qwen3_trace(eng._h, None, 0, ctypes.byref(n)))
    buf = np.zeros(n.value, np.uint64)
    _lib.check(eng.lib.xpu_qwen3_trace(eng._h, buf.ctypes.data, n.value, ctypes.byref(n)))
    events = 1 + 24 * L + 2
    t = buf.reshape(-1, events).astype(np.int64)
    t -= t[:, 0].min()
    out = [f"step span {t[:, -1].max() / 1e3:.1f} us over {t.shape[0]} CTAs; "
           f"per layer {(t[:, 1 + 24 * L] - t[:, 1]).max() / L / 1e3:.1f} us"]
    for ph in range(6):
        cells = []
        for k in range(4):
            e = np.array([1 + 24 * l + 4 * ph + k for l in range(L)])
            dur = t[:, e] - t[:, e - 1]
            cells.append(f"{PARTS[k]} {dur.mean() / 1e3:6.2f}/{dur.max(axis=0).mean() / 1e3:6.2f}")
        out.append(f"{PHASES[ph]:8s} " + "  ".join(cells))
    lm = t[:, -1] - t[:, -3]
    out.append(f"lm_head  total {lm.mean() / 1e3:.1f}/{lm.max() / 1e3:.1f} us (mean/max over CTAs)")
    return out


def prefill_profile(args) -> None:
    import time

    import torch

    from .qwen3 import Qwen3Engine
    from .qwen3_config import PRESETS

    shape = PRESETS[args.preset]
    prompt = [int(t) for t in np.random.default_rng(7).integers(0, shape.vocab, args.prefill)]
    with Qwen3Engine(shape, args.prefill + 8) as eng:
        eng.init_synthetic(1)
        eng.prefill_dense(prompt)
        eng.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        t0 = time.perf_counter()
        nxt = eng.prefill_dense(prompt)
        dt = time.perf_counter() - t0
        torch.cuda.cudart().cudaProfilerStop()
    print(f"{args.preset}: dense prefill of {args.prefill} tokens {dt * 1e3:.2f} ms "
          f"({args.prefill / dt:.0f} tok/s), next token {nxt}")


def batch_profile(args) -> None:
    if args.trace:
        os.environ["XPU_BATCH_TRACE"] = "1"
    import torch

    from .qwen3 import Qwen3Engine
    from .qwen3_config import PRESETS

    shape, B = PRESETS[args.preset], args.batch
    eng = Qwen3Engine(shape, args.context + args.warm + 8, max_batch=B)
    eng.init_synthetic(2026)
    rng = np.random.default_rng(7)
    prompts = [[int(t) for t in rng.integers(0, shape.vocab, size=args.context)] for _ in range(B)]
    eng.batch_generate(prompts, 1)  # prefill: every sequence at `context` positions
    eng.batch_enqueue_steps(args.warm)
    eng.synchronize()
    if args.trace:
        eng.batch_trace()  # reset
    torch.cuda.cudart().cudaProfilerStart()
    eng.batch_enqueue_steps(1)
    eng.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    _, pos, err = eng.batch_state(B)
    print(f"{args.preset}: batch {B}, positions {pos[0]}, error {err}, kernels/step {eng.batch_kernels_per_step()}")
    if args.trace:
        tr = eng.batch_trace().astype(np.int64)[:eng.batch_kernels_per_step()]
        names = ["embed"] + ["qkv", "attention", "o_proj", "gate_up", "down"] * shape.layers + ["lm_head", "argmax"]
        t0, prev = tr[0, 0], tr[0, 0]
        print(f"step span {(tr[:, 2].max() - t0) / 1e3:.1f} us")
        acc: dict[str, np.ndarray] = {}
        for name, row in zip(names, tr):
            start, wmax, end, wmin, smax, first, last, epi = row
            a = acc.setdefault(name, np.zeros(6))
            a[0] += 1
            a[1] += (end - prev) / 1e3
            a[2] += (wmin - prev) / 1e3
            if first:
                a[3] += (first - wmin) / 1e3
                a[4] += (last - wmin) / 1e3
                a[5] += (epi - last) / 1e3
            if name == "attention" and first:
                # attention marks: heads finished, probabilities ready, output accumulated
                att = acc.setdefault("attention phases", np.zeros(6))
                att[0] += 1
                att[1] += (first - wmin) / 1e3
                att[2] += (last - first) / 1e3
                att[3] += (epi - last) / 1e3
                att[4] += (end - epi) / 1e3
            prev = end
        for name, a in acc.items():
            c = a[0]
            if name == "attention phases":
                print(f"attention phases (last CTA, after the wait): heads {a[1] / c:6.2f} us, scores + softmax "
                      f"{a[2] / c:6.2f}, p.v {a[3] / c:6.2f}, output {a[4] / c:6.2f}")
                continue
            print(f"{name:9s} x{int(c):3d} critical {a[1] / c:7.2f} us | wait returns {a[2] / c:5.2f} after the "
                  f"previous end | first stage {a[3] / c:6.2f}, final accumulator {a[4] / c:6.2f} after the wait | "
                  f"epilogue tail {a[5] / c:5.2f}")
    eng.close()


if __name__ == "__main__":
    main()
