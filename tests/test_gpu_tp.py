"""Tensor-parallel DiT on 2 GPUs (one process per GPU; the partial projections summed by the LayerNorm kernel over
peer memory, by the same reduce-scatter + row-sharded LayerNorm + all-gather over peer memory or through NCCL, or by
an NCCL all-reduce in bf16 or fp32) against the unsharded CPU oracle: velocity cosine >= 0.999;
the peer forms and NCCL's bf16 all-reduce / reduce-scatter agree bit for bit at 2 ranks. Needs two GPUs; skipped
otherwise.

The bounded wait of the fused kernel is checked on one GPU: a signal pad that no rank writes makes the wait run out,
the kernel records the error and returns, and the context stays usable."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

_PORTS = iter(range(29800 + (os.getpid() % 40) * 40, 29800 + (os.getpid() % 40) * 40 + 40))


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
        model.close()
        twin = {"peer": "bf16", "peer_rs": "rs"}.get(reduce_dtype)
        if twin:     # the same step through NCCL (all-reduce / reduce-scatter, bf16): identical at two ranks
            nccl = dit.DiT(cfg, dit.shard_weights(w, cfg, rank, world), device=f"cuda:{rank}",
                           tp=(rank, world, dist.group.WORLD), reduce_dtype=twin)
            v2 = nccl.forward(torch.from_numpy(lat), torch.from_numpy(txt), 0.5).float().cpu().numpy()
            if rank == 0:
                q.put(bool(np.array_equal(v, v2)))
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


@pytest.mark.parametrize("reduce_dtype", ["peer", "peer_rs", "rs", "bf16", "fp32"])
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
    got = [q.get(timeout=10) for _ in range(2 if reduce_dtype in ("peer", "peer_rs") else 1)]
    cos = next(g for g in got if not isinstance(g, bool))
    assert cos >= 0.999, f"TP-2 velocity cosine {cos:.6f}"
    if reduce_dtype in ("peer", "peer_rs"):
        assert next(g for g in got if isinstance(g, bool)), "peer sum differs from NCCL's bf16 reduction"


@pytest.mark.parametrize("reduce_dtype", ["peer_rs", "rs", "bf16"])
def test_tp4_dit_matches_oracle(reduce_dtype):
    """The reductions that run on more than 2 GPUs, at 4 ranks (a 4-head, 2-block toy whose 256 rows shard into
    blocks of 64): velocity cosine >= 0.999 against the unsharded CPU oracle. Needs four GPUs; skipped otherwise."""
    import torch
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = next(_PORTS)
    cfg = dict(hidden=512, heads=4, ffn=1024, blocks=2, text=64, image=192, grid=(12, 16))
    procs = [ctx.Process(target=_worker, args=(r, 4, port, q, cfg, reduce_dtype)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = [q.get(timeout=10) for _ in range(2 if reduce_dtype == "peer_rs" else 1)]
    cos = next(g for g in got if not isinstance(g, bool))
    assert cos >= 0.999, f"TP-4 velocity cosine {cos:.6f}"


def test_ln_mod_tp_wait_runs_out_cleanly():
    """rl_ln_mod_tp with W = 2 and a pad the other rank never writes: after its bounded wait (about two seconds) the
    kernel records the timeout and returns without writing; rl_device_status reports it, and the next launch runs."""
    import torch
    from redline_tiny_b200 import _lib as L
    from redline_tiny_b200 import ops
    dev = torch.device("cuda", 0)
    M, D = 16, 256
    x = torch.randn(M, D, device=dev).to(torch.bfloat16)
    part = torch.randn(M, D, device=dev).to(torch.bfloat16)
    # the partials in the projection GEMM's chunk layout: 16-row x 32-column chunks of 512 values
    chunked = part.view(M // 16, 16, D // 32, 32).permute(0, 2, 1, 3).contiguous()
    parts = torch.tensor([chunked.data_ptr(), chunked.data_ptr()], dtype=torch.int64, device=dev)
    pad = torch.zeros(2, dtype=torch.int64, device=dev)
    params = torch.ones(2, 2, D, device=dev).to(torch.bfloat16)
    xo = torch.full((M, D), 7.0, device=dev).to(torch.bfloat16)
    y = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream
    L.call("rl_ln_mod_tp", x.data_ptr(), parts.data_ptr(), 2, pad.data_ptr(), 0, 1, params.data_ptr(), M, D, 0,
           xo.data_ptr(), y.data_ptr(), None, s)
    with pytest.raises(L.RedlineError):
        ops.device_status()
    assert bool((xo.float() == 7.0).all()), "the kernel wrote x_out after its wait ran out"
    # the pad now holds the peer's epoch: the same launch completes and sums the two partials
    pad[1] = 1
    L.call("rl_ln_mod_tp", x.data_ptr(), parts.data_ptr(), 2, pad.data_ptr(), 0, 1, params.data_ptr(), M, D, 0,
           xo.data_ptr(), y.data_ptr(), None, s)
    ops.device_status()
    br = (part.float() * 2).to(torch.bfloat16).float()
    ref = (x.float() + br).to(torch.bfloat16).float()
    assert torch.equal(xo.float(), ref)


def test_tp_wait_runs_out_cleanly():
    """rl_tp_wait on a pad that nothing writes: the wait runs out (about two seconds), the error is reported and the
    next launch runs; with the epochs present it passes."""
    import torch
    from redline_tiny_b200 import _lib as L
    from redline_tiny_b200 import ops
    dev = torch.device("cuda", 0)
    pad = torch.zeros(4, dtype=torch.int64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    L.call("rl_tp_wait", pad.data_ptr(), 4, 1, 3, s)
    with pytest.raises(L.RedlineError):
        ops.device_status()
    pad.fill_(3)
    L.call("rl_tp_wait", pad.data_ptr(), 4, 1, 3, s)
    ops.device_status()


def _chunked(t):
    """(M, D) -> the partial chunk layout: 16-row x 32-column chunks of 512 values, chunk-row-major."""
    M, D = t.shape
    return t.view(M // 16, 16, D // 32, 32).permute(0, 2, 1, 3).contiguous()


def test_scatter_gemm_and_rs_layernorm_one_gpu():
    """The peer reduce-scatter pieces on one GPU with W = 2 (both ranks' buffers local): rl_linear_bfp16_scatter
    stores rows [0, R) and [R, 2R) in the chunk layout of each block, bit-equal to rl_linear_bfp16_partial's; and
    rl_ln_mod_tp_rs over one block equals rl_ln_mod_tp on the same rows, bit for bit, in every y destination."""
    import torch
    from redline_tiny_b200 import _lib as L
    from redline_tiny_b200 import ops
    dev = torch.device("cuda", 0)
    s = torch.cuda.current_stream().cuda_stream
    M, K, N, W = 512, 256, 384, 2
    R = M // W
    g = torch.Generator(device=dev).manual_seed(3)
    _, x = ops.quantize_bfp16(torch.randn(M, K, generator=g, device=dev), want_bytes=False)
    w = ops.PackedWeight.from_float(torch.randn(K, N, generator=g, device=dev) * 0.05)
    full = torch.empty(M * N, dtype=torch.bfloat16, device=dev)
    L.call("rl_linear_bfp16_partial", x.data_ptr(), M, K, w.native.data_ptr(), N, full.data_ptr(), None, s)
    blocks = [torch.full((R * N,), 5.0, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    dsts = torch.tensor([b.data_ptr() for b in blocks], dtype=torch.int64, device=dev)
    L.call("rl_linear_bfp16_scatter", x.data_ptr(), M, K, w.native.data_ptr(), N, dsts.data_ptr(), W, R, s)
    ops.device_status()
    for o in range(W):      # block o of the full partial is its rows' chunks: a contiguous range of chunk rows
        assert torch.equal(blocks[o].view(torch.int16), full[o * R * N:(o + 1) * R * N].view(torch.int16))
    # the LayerNorm of rank 1's rows from two partials
    D = N
    xin = torch.randn(R, D, generator=g, device=dev).to(torch.bfloat16)
    p0 = torch.randn(R, D, generator=g, device=dev).to(torch.bfloat16)
    p1 = torch.randn(R, D, generator=g, device=dev).to(torch.bfloat16)
    parts = [_chunked(p0), _chunked(p1)]
    parts_t = torch.tensor([p.data_ptr() for p in parts], dtype=torch.int64, device=dev)
    params = (1 + 0.1 * torch.randn(2, 2, D, generator=g, device=dev)).to(torch.bfloat16)
    pad = torch.tensor([4, 0], dtype=torch.int64, device=dev)       # rank 1 waits for rank 0's epoch 4
    xo_ref = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    y_ref = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    L.call("rl_ln_mod_tp", xin.data_ptr(), parts_t.data_ptr(), 2, pad.data_ptr(), 1, 4, params.data_ptr(), R, D, 40,
           xo_ref.data_ptr(), y_ref.data_ptr(), None, s)
    xo = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    outs = [torch.zeros(M, D, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    y_dsts = torch.tensor([o[R:].data_ptr() for o in outs], dtype=torch.int64, device=dev)
    L.call("rl_ln_mod_tp_rs", xin.data_ptr(), parts_t.data_ptr(), 2, pad.data_ptr(), 1, 4, params.data_ptr(), R, D,
           40, xo.data_ptr(), y_dsts.data_ptr(), s)
    ops.device_status()
    assert torch.equal(xo.view(torch.int16), xo_ref.view(torch.int16))
    for o in outs:
        assert torch.equal(o[R:].view(torch.int16), y_ref.view(torch.int16))
        assert not o[:R].float().any(), "rows of the other rank were written"
