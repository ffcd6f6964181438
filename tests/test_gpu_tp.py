"""Tensor-parallel DiT on 2 GPUs (one process per GPU, NCCL all-reduce of the partial projections in bf16 and in
fp32) against the unsharded CPU oracle: velocity cosine >= 0.999. Needs two GPUs; skipped otherwise."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

_PORTS = iter(range(29800 + (os.getpid() % 40) * 10, 29800 + (os.getpid() % 40) * 10 + 10))


def _worker(rank, world, port, q, blocks_cfg, reduce_dtype):
    import datetime
    import torch
    import torch.distributed as dist
    from redline_tiny_b200 import dit, ops
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        cfg = dit.DiTConfig(**blocks_cfg)
        w = dit.random_weights(cfg, seed=5, device=f"cuda:{rank}")
        model = dit.DiT(cfg, dit.shard_weights(w, cfg, rank, world), device=f"cuda:{rank}",
                        tp=(rank, world, dist.group.WORLD), reduce_dtype=reduce_dtype)
        rng = np.random.default_rng(5)
        lat = rng.standard_normal((cfg.image, cfg.latent_ch)).astype(np.float32)
        txt = rng.standard_normal((cfg.text, cfg.hidden)).astype(np.float32)
        v = model.forward(torch.from_numpy(lat), torch.from_numpy(txt), 0.5).float().cpu().numpy()
        ops.device_status()
        if rank == 0:
            from oracle import dit_oracle as DO
            from redline_tiny_b200 import host_glue as HG
            wc = {"blocks": [{k: t.cpu() for k, t in b.items()} for b in w["blocks"]], "host": w["host"],
                  "img_in": w["img_in"].cpu(), "proj_out": w["proj_out"].cpu()}
            ref = DO.forward(cfg, DO.prepare(wc), lat, txt, 0.5, HG)
            a, b = v.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
            q.put(float(a @ b / np.sqrt((a @ a) * (b @ b))))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("reduce_dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("blocks_cfg", [dict(hidden=256, heads=2, ffn=512, blocks=2, text=64, image=192, grid=(12, 16)),
                                        dict(blocks=1)])
def test_tp2_dit_matches_oracle(blocks_cfg, reduce_dtype):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = next(_PORTS)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, blocks_cfg, reduce_dtype)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    cos = q.get(timeout=10)
    assert cos >= 0.999, f"TP-2 velocity cosine {cos:.6f}"
