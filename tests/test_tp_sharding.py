"""Tensor-parallel DiT sharding on CPU: two gloo ranks each run the oracle block math on their shard
(redline_tiny_b200.dit.shard_weights: heads for QKV / attention / out-projection, FFN units for up / down) and add
the partial projection outputs with an all-reduce; the result must equal the unsharded oracle (only the order of
the float32 additions differs)."""

import os

import numpy as np
import pytest


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle import dit_oracle as DO
    from redline_tiny_b200 import dit, host_glue as HG
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = dit.DiTConfig(hidden=256, heads=2, ffn=512, blocks=2, text=64, image=192, grid=(12, 16))
        w = dit.random_weights(cfg, seed=3, device="cpu")
        rng = np.random.default_rng(3)
        lat = rng.standard_normal((cfg.image, cfg.latent_ch)).astype(np.float32)
        txt = rng.standard_normal((cfg.text, cfg.hidden)).astype(np.float32)

        def reduce(c):
            t = torch.from_numpy(np.ascontiguousarray(c, np.float32))
            dist.all_reduce(t)
            return t.numpy()
        v_tp = DO.forward(cfg, DO.prepare(dit.shard_weights(w, cfg, rank, world)), lat, txt, HG.SIGMAS[2], HG,
                          reduce=reduce)
        v_full = DO.forward(cfg, DO.prepare(w), lat, txt, HG.SIGMAS[2], HG)
        a, b = v_tp.astype(np.float64).ravel(), v_full.astype(np.float64).ravel()
        q.put((rank, float(a @ b / np.sqrt((a @ a) * (b @ b))), float(np.abs(a - b).max() / np.abs(b).max())))
    finally:
        dist.destroy_process_group()


def test_tp2_oracle_equals_unsharded():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, cos, err in res:
        assert cos > 0.9999 and err < 2e-2, f"rank {rank}: cosine {cos:.6f} max-rel {err:.3e}"


def test_shard_shapes():
    from redline_tiny_b200 import dit
    cfg = dit.DiTConfig(blocks=1)
    import torch
    w = {"blocks": [{"qkv": torch.zeros(3072, 9216), "o": torch.zeros(3072, 3072), "gate": torch.zeros(12288, 3072),
                     "proj": torch.zeros(12288, 3072), "down": torch.zeros(12288, 3072), "norm_q": torch.zeros(128),
                     "norm_k": torch.zeros(128)}], "host": {}, "img_in": None, "proj_out": None}
    for world in (2, 4, 8):
        s = dit.shard_weights(w, cfg, world - 1, world)["blocks"][0]
        assert s["qkv"].shape == (3072, 3 * 3072 // world)
        assert s["o"].shape == (3072 // world, 3072)
        assert s["gate"].shape == (12288 // world, 3072) and s["down"].shape == (12288 // world, 3072)
    with pytest.raises(AssertionError):
        dit.shard_weights(w, cfg, 0, 5)


def test_reduction_choice_is_checked():
    """DiT's reduce_dtype is checked before anything is allocated; the peer reduction is built for exactly 2 ranks."""
    import pytest
    from redline_tiny_b200 import dit, tp
    with pytest.raises(ValueError, match="reduce_dtype"):
        dit.DiT(dit.DiTConfig(blocks=1), {}, device="cpu", reduce_dtype="fp16")
    with pytest.raises(ValueError, match="2 ranks"):
        tp.PeerReduce(None, 0, 4, 64, 256, "cpu")
