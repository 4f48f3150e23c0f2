"""Profile one Qwen3 decode step (the launch that ncu captures, or a phase trace).

    python -m xpu_playground_b200.profile_step --preset qwen3-8b-l2 --context 2048 --warm 2
    python -m xpu_playground_b200.profile_step --preset qwen3-8b --context 2048 --trace

The default run builds a seeded synthetic model, places the decode state at
`--context` cached positions (the KV cache contents do not change the work),
and runs `--warm` + 1 decode steps, so that the step to capture under
`ncu -k regex:k_step -s <warm> -c 1` is the last one. Weight initialisation
launches one fill kernel per tensor before that.

Under torchrun the ranks run one tensor-parallel engine and rank 0 reports:

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        -m xpu_playground_b200.profile_step --preset qwen3-8b --trace

--trace re-runs with XPU_STEP_TRACE=1 and prints, per phase of the persistent
step, the mean/max over CTAs of the time spent staging the activation,
streaming its items, finishing (arrivals and epilogues) and in the grid
barrier, averaged over layers.
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
    args = ap.parse_args()
    if args.trace:
        os.environ["XPU_STEP_TRACE"] = "1"

    from . import _lib
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
    if world > 1:
        dist.barrier()
        if rank != 0:
            dist.barrier()
            eng.close()
            dist.destroy_process_group()
            return
    print(f"{args.preset}: position {pos}, last token {tok}, error {err}, tp {world}, "
          f"kernels/step {eng.info().kernels_per_step}, fill launches {len(shape.tensor_names())}")
    if not args.trace:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    n = ctypes.c_uint32()
    _lib.check(eng.lib.xpu_qwen3_trace(eng._h, None, 0, ctypes.byref(n)))
    buf = np.zeros(n.value, np.uint64)
    _lib.check(eng.lib.xpu_qwen3_trace(eng._h, buf.ctypes.data, n.value, ctypes.byref(n)))
    L = shape.layers
    events = 1 + 24 * L + 2
    t = buf.reshape(-1, events).astype(np.int64)
    t -= t[:, 0].min()
    print(f"step span {t[:, -1].max() / 1e3:.1f} us over {t.shape[0]} CTAs; "
          f"per layer {(t[:, 1 + 24 * L] - t[:, 1]).max() / L / 1e3:.1f} us")
    for ph in range(6):
        cells = []
        for k in range(4):
            e = np.array([1 + 24 * l + 4 * ph + k for l in range(L)])
            dur = t[:, e] - t[:, e - 1]
            cells.append(f"{PARTS[k]} {dur.mean() / 1e3:6.2f}/{dur.max(axis=0).mean() / 1e3:6.2f}")
        print(f"{PHASES[ph]:8s} " + "  ".join(cells))
    lm = t[:, -1] - t[:, -3]
    print(f"lm_head  total {lm.mean() / 1e3:.1f}/{lm.max() / 1e3:.1f} us (mean/max over CTAs)")
    if world > 1:
        dist.barrier()
        eng.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
