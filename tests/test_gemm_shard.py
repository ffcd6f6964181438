"""The N-split standalone GEMM on CPU: the column-shard arithmetic of the C ABI (rl_weights_shard, no device
touched) and two gloo ranks that each run the oracle GEMM on their contiguous byte range of the reference's pack_b
stream (redline/pack_weights.py:72-79; strips of 128 columns whole, N-tile outer: redline/npu_layouts.py:11-16) and
all-gather the column blocks; the result must equal the unsharded oracle GEMM bit for bit (each column's dot
products are the same float32 operations in either case)."""

import os

import numpy as np
import pytest


@pytest.fixture(scope="module")
def ops():
    from redline_tiny_b200 import build
    build.build()
    from redline_tiny_b200 import ops as o
    return o


def test_shard_ranges_tile_the_packed_stream(ops):
    K, N = 3072, 12288
    total = K * N // 8 * 9
    for world in (1, 2, 4, 8):
        end_b, end_n = 0, 0
        for r in range(world):
            n0, cols, off, count = ops.weights_shard(K, N, r, world)
            assert (n0, off) == (end_n, end_b) and cols == N // world
            assert count == K * cols // 8 * 9 and off % 9216 == 0
            end_n, end_b = n0 + cols, off + count
        assert (end_n, end_b) == (N, total)


def test_shard_rejects_uneven_splits(ops):
    from redline_tiny_b200 import _lib as L
    with pytest.raises(L.RedlineError, match="128 \\* world"):
        ops.weights_shard(3072, 384, 0, 2)
    with pytest.raises(L.RedlineError, match="rank"):
        ops.weights_shard(3072, 12288, 8, 8)
    with pytest.raises(L.RedlineError):
        ops.weights_shard(100, 12288, 0, 2)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle import bfp16_oracle as O
    from redline_tiny_b200 import ops
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, K, N = 96, 256, 1024
        rng = np.random.default_rng(4)
        x = rng.standard_normal((M, K)).astype(np.float32)
        W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        packed = O.pack_b(W)
        n0, cols, off, count = ops.weights_shard(K, N, rank, world)
        _, xd = O.quantize_rows(x)
        mine = O.linear(xd, O.unpack_b(packed[off:off + count], K, cols)).astype(np.float32)
        parts = [torch.empty(M, cols) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine)))
        got = torch.cat(parts, 1).numpy()
        full = O.linear(xd, O.unpack_b(packed, K, N)).astype(np.float32)
        q.put((rank, n0, bool(np.array_equal(got, full))))
    finally:
        dist.destroy_process_group()


def test_two_rank_n_split_equals_unsharded_oracle():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 150
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert [r[1] for r in res] == [0, 512]
    assert all(r[2] for r in res), res
