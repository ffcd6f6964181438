"""Per-launch times of one tensor-parallel DiT denoise step (config 4), for each requested reduction - where the time
of a block goes and what the out- and down-projection reductions cost. One process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29631 \\
        -m redline_tiny_b200.tp_phases peer bf16

Each rank records a CUDA event after every launch of a step (after warm-up steps) and prints, for block 10, the time
between consecutive events per launch (microseconds), and for the whole step the total per entry point. The events
add a little to the step; compare modes within one run. Random-init weights, seeded synthetic inputs.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

from . import _lib as L
from . import dit, ops


def main():
    modes = sys.argv[1:] or ["auto"]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        cfg = dit.DiTConfig()
        lat = torch.randn((cfg.image, cfg.latent_ch), generator=torch.Generator(device=dev).manual_seed(7), device=dev)
        txt = torch.randn((cfg.text, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(8), device=dev)
        for mode in modes:
            w = dit.random_weights(cfg, seed=1000)
            model = dit.DiT(cfg, dit.shard_weights(w, cfg, rank, world), device=dev, tp=(rank, world, dist.group.WORLD),
                            reduce_dtype=mode)
            del w
            for _ in range(3):
                model.denoise_step(lat, txt, 3)
            torch.cuda.synchronize()
            dist.barrier()
            marks = []

            def mark(name):
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                marks.append((name, e))

            call, all_reduce = L.call, dist.all_reduce

            def timed_call(name, *a):
                r = call(name, *a)
                mark(name[3:] if name.startswith("rl_") else name)
                return r

            def timed_all_reduce(*a, **k):
                r = all_reduce(*a, **k)
                mark("nccl_all_reduce")
                return r
            L.call, dist.all_reduce = timed_call, timed_all_reduce
            try:
                mark("start")
                model.denoise_step(lat, txt, 3)
                torch.cuda.synchronize()
            finally:
                L.call, dist.all_reduce = call, all_reduce
            seq = [(n1, e0.elapsed_time(e1) * 1e3) for (_, e0), (n1, e1) in zip(marks, marks[1:])]
            totals = {}
            for n, us in seq:
                t = totals.setdefault(n, [0, 0.0])
                t[0] += 1
                t[1] += us
            starts = [i for i, (n, _) in enumerate(seq) if n == "qkv_post"]
            block = seq[starts[10] - 1:starts[11] - 1] if len(starts) > 11 else []
            step_ms = marks[0][1].elapsed_time(marks[-1][1])
            print(f"rank {rank} {mode} ({model.reduce_dtype}): step {step_ms:.2f} ms; block 10 (us): "
                  + ", ".join(f"{n} {us:.1f}" for n, us in block), flush=True)
            print(f"rank {rank} {mode}: per entry point (ms / launches): "
                  + ", ".join(f"{n} {t[1] / 1e3:.2f}/{t[0]}" for n, t in totals.items()), flush=True)
            ops.device_status()
            model.close()
            del model
            torch.cuda.empty_cache()
            dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
