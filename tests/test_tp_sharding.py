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


def test_peer_rs_layout():
    """The peer reduce-scatter's buffers for 2 to 8 ranks at config 4 (and a toy size): inside each rank's
    allocation, 256-byte aligned, non-overlapping; every rank's scatter destination for owner o is that owner's
    receive buffer of the sender; the all-gather destinations are the sender's rows of every operand."""
    from redline_tiny_b200 import tp
    for M, D in ((4352, 3072), (256, 256)):
        for W in range(2, 9):
            if M % W or (M // W) % 16:
                continue
            bases = [(1 + r) << 40 for r in range(W)]            # far apart: any spill into a neighbour shows
            lays = [tp.peer_rs_layout(M, D, W, r, bases) for r in range(W)]
            L0 = lays[0]
            R = M // W
            assert L0["R"] == R and L0["recv_bytes"] >= R * D * 2
            regions = [(s * W + src) * L0["recv_bytes"] for s in range(2) for src in range(W)]
            ends = [o + R * D * 2 for o in regions]
            assert all(e <= n for e, n in zip(ends, regions[1:] + [L0["a_off"]]))
            assert L0["a_off"] + M * D * 2 <= L0["pad_off"] and L0["pad_off"] + 3 * W * 8 <= L0["bytes"]
            for r, lay in enumerate(lays):
                for s in range(2):
                    for o in range(W):
                        assert lay["dsts"][s][o] == lays[o]["parts"][s][r]      # sender r -> owner o, slot s
                        assert lay["dsts"][s][o] % 256 == 0
                        assert bases[o] <= lay["dsts"][s][o] < bases[o] + L0["a_off"]
                for o in range(W):
                    assert lay["y_dsts"][o] == bases[o] + L0["a_off"] + r * R * D * 2
                    assert lay["pads"][o] == bases[o] + L0["pad_off"]
    import pytest
    with pytest.raises(ValueError):
        tp.peer_rs_layout(4352, 3072, 5, 0, [0] * 5)
