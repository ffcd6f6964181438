"""GPU parity of the packed-weight tcgen05 GEMM (and its SwiGLU epilogue) against the CPU oracle:
C = from_bfp16(Xq) @ from_bfp16(Wq) (+ bias) in float32 (oracle/bfp16_oracle.linear).

Tolerances (max-rel = max|got - ref| / max|ref|, the statistic of redline/run_ln.py:74-79):
  fp32 output:  <= 1e-4 against the fp32 oracle (only the accumulation order differs);
  bf16 output:  <= 2e-3 + 2^-8 against the fp32 oracle: the north-star bound plus the output's own rounding to bf16,
                which alone moves a value by up to 2^-8 of max|ref|;
  SwiGLU:       <= 2e-3 against the oracle's H rounded to bfp16 (blocks of 8 along F), like the reference's flush."""

import numpy as np
import pytest

from oracle import bfp16_oracle as O

pytestmark = pytest.mark.gpu

VARIANTS = [1, 2, 3, 4]   # 1-SM with A in shared memory / TMEM, 2-SM pair with A in shared memory / TMEM (pairs need N % 256 == 0)
BF16_OUT_TOL = 2e-3 + 2.0 ** -8


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import ops
    assert torch.cuda.is_available()
    return torch, ops, torch.device("cuda:0")


def _case(M, K, N, seed=0, bias=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    b = O.bf16_round((rng.standard_normal(N) * 0.01).astype(np.float32)) if bias else None
    return x, W, b


def _skip_unpairable(variant, N):
    if variant in (3, 4) and N % 256:
        pytest.skip("the pair kernel covers N % 256 == 0 (others use the 1-SM kernel)")


def _run(env, x, W, b, out_dtype, variant, rows=None):
    torch, ops, dev = env
    M, K = x.shape
    N = W.shape[1]
    _skip_unpairable(variant, N)
    prev = ops.set_gemm_variant(variant)
    try:
        _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
        w = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(W)).to(dev), K, N)
        bt = None if b is None else torch.from_numpy(b).to(dev).to(torch.bfloat16)
        c = ops.linear_bfp16(dq, w, bias=bt, out_dtype=out_dtype)
        ops.device_status()
    finally:
        ops.set_gemm_variant(prev)
    got = c.float().cpu().numpy()
    sel = slice(None) if rows is None else rows
    _, xd = O.quantize_rows(x[sel])
    ref = O.linear(xd, O.unpack_b(O.pack_b(W), K, N), b)
    return got[sel], ref


def _diag(got, ref):
    bad = np.abs(got - ref) > 2e-3 * np.abs(ref).max()
    if not bad.any():
        return "ok"
    r, c = np.nonzero(bad)
    return (f"{bad.sum()} bad of {bad.size}; rows {np.unique(r)[:16]} ({len(np.unique(r))} distinct), "
            f"cols {np.unique(c)[:16]} ({len(np.unique(c))} distinct); corr {O.corr(got, ref):.5f}")


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("M,K,N", [(128, 128, 256), (256, 64, 128), (1, 64, 128), (300, 192, 384),
                                   (512, 4096, 256)])
def test_linear_small(env, variant, M, K, N):
    torch = env[0]
    x, W, b = _case(M, K, N)
    got, ref = _run(env, x, W, b, torch.float32, variant)
    err = O.max_rel(got, ref)
    assert err <= 1e-4, f"max-rel {err:.3e}: {_diag(got, ref)}"


@pytest.mark.parametrize("variant", VARIANTS)
def test_linear_bf16_out_no_bias(env, variant):
    torch = env[0]
    x, W, _ = _case(384, 256, 512, seed=2, bias=False)
    got, ref = _run(env, x, W, None, torch.bfloat16, variant)
    err = O.max_rel(got, ref)
    assert err <= BF16_OUT_TOL, f"max-rel {err:.3e}: {_diag(got, ref)}"


@pytest.mark.parametrize("variant", VARIANTS)
def test_linear_config1_full_size(env, variant):
    """Benchmark config 1 (DiT FFN up-projection): X[4352, 3072] ~ N(0,1), W[3072, 12288] ~ N(0, 0.02), bias
    ~ N(0, 0.01), bf16 out. The oracle runs on a sample of 256 rows (every M tile, first and last rows)."""
    torch = env[0]
    x, W, b = _case(4352, 3072, 12288, seed=0)
    rows = np.unique(np.concatenate([np.arange(0, 4352, 17), [0, 255, 256, 4095, 4351]]))
    got, ref = _run(env, x, W, b, torch.bfloat16, variant, rows=rows)
    err = O.max_rel(got, ref)
    assert err <= BF16_OUT_TOL, f"max-rel {err:.3e}: {_diag(got, ref)}"


def _swiglu_case(M, K, F, seed=5):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wg = (rng.standard_normal((F, K)) * 0.02).astype(np.float32)
    wp = (rng.standard_normal((F, K)) * 0.02).astype(np.float32)
    return x, O.interleave_up(wg, wp)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("M,K,F", [(128, 128, 128), (300, 256, 256), (512, 4096, 1024)])
def test_swiglu_up(env, variant, M, K, F):
    torch, ops, dev = env
    _skip_unpairable(variant, 2 * F)
    x, Bup = _swiglu_case(M, K, F)
    prev = ops.set_gemm_variant(variant)
    try:
        _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
        w = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(Bup)).to(dev), K, 2 * F, swiglu=True)
        h = ops.swiglu_up(dq, w)
        ops.device_status()
    finally:
        ops.set_gemm_variant(prev)
    got = h.float().cpu().numpy()
    _, xd = O.quantize_rows(x)
    c = O.linear(xd, O.unpack_b(O.pack_b(Bup), K, 2 * F))
    href = O.swiglu_from_interleaved(c)
    _, href_q = O.quantize_rows(href)          # the reference rounds H to bfp16 for the down GEMM
    err = O.max_rel(got, href_q)
    assert err <= 2e-3, f"max-rel {err:.3e}: {_diag(got, href_q)}"
    # the same bfp16 values almost everywhere (blocks whose rounding sits on a tie can differ by one step)
    assert np.mean(got == href_q) > 0.99


def test_linear_split_k_small_grid(env):
    """rl_linear_bfp16_ws: 32 pair tiles with 96 K steps each run as 2 K ranges (fp32 partials in the workspace, then
    a reduction adding them and the bias); matches the oracle on sampled rows and the unsplit kernel up to fp32
    summation order, and a too-small workspace falls back to the unsplit kernel."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    M, K, N = 512, 6144, 4096
    x, W, b = _case(M, K, N, seed=11)
    _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    w = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(W)).to(dev), K, N)
    bt = torch.from_numpy(b).to(dev).to(torch.bfloat16)
    need = L.lib().rl_linear_bfp16_workspace(M, K, N, L.RL_EPI_BIAS)
    # 32 pair tiles x 2 ranges need 64 resident clusters (74 on a full B200; fewer when the GPC layout leaves SMs
    # unpaired, and then the split is not taken)
    if L.lib().rl_gemm_pair_clusters() < 64:
        pytest.skip(f"only {L.lib().rl_gemm_pair_clusters()} resident pair clusters")
    assert need == 2 * M * N * 4
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    rows = np.r_[0:16, 500:512]
    _, xd = O.quantize_rows(x[rows])
    ref = O.linear(xd, O.unpack_b(O.pack_b(W), K, N), b)
    for dt, code, tol, agree in ((torch.bfloat16, L.RL_BF16, BF16_OUT_TOL, 2.0 ** -7), (torch.float32, L.RL_F32, 2e-3, 1e-5)):
        c = torch.empty((M, N), dtype=dt, device=dev)
        L.call("rl_linear_bfp16_ws", dq.data_ptr(), M, K, w.native.data_ptr(), N, bt.data_ptr(), L.RL_EPI_BIAS,
               c.data_ptr(), code, ws.data_ptr(), need, s)
        u = torch.empty((M, N), dtype=dt, device=dev)
        L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), N, bt.data_ptr(), L.RL_EPI_BIAS,
               u.data_ptr(), code, s)
        ops.device_status()
        got = c.float().cpu().numpy()[rows]
        assert O.max_rel(got, ref) <= tol, _diag(got, ref)
        assert (c.float() - u.float()).abs().max().item() <= agree * u.float().abs().max().item()
    c = torch.empty((M, N), dtype=torch.float32, device=dev)
    L.call("rl_linear_bfp16_ws", dq.data_ptr(), M, K, w.native.data_ptr(), N, bt.data_ptr(), L.RL_EPI_BIAS,
           c.data_ptr(), L.RL_F32, ws.data_ptr(), need - 16, s)
    unsplit = torch.empty((M, N), dtype=torch.float32, device=dev)
    L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), N, bt.data_ptr(), L.RL_EPI_BIAS,
           unsplit.data_ptr(), L.RL_F32, s)
    assert torch.equal(c, unsplit)


def test_linear_grouped_tile_order(env):
    """Pair tiles walk groups of activation tiles sized to ~40 MB of X: at K = 12288 a group is 6 tiles at most, so
    19 activation tiles (ragged M) form groups of 5, 5, 5 and 4; every tile is computed once and correctly (oracle
    on rows of every group)."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    M, K, N = 4800, 12288, 512
    x, W, b = _case(M, K, N, seed=31)
    _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    w = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(W)).to(dev), K, N)
    bt = torch.from_numpy(b).to(dev).to(torch.bfloat16)
    c = torch.empty((M, N), dtype=torch.float32, device=dev)
    L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), N, bt.data_ptr(), L.RL_EPI_BIAS,
           c.data_ptr(), L.RL_F32, torch.cuda.current_stream().cuda_stream)
    ops.device_status()
    rows = np.unique(np.r_[0:4, 1275:1285, 2555:2565, 3835:3845, 4790:4800])
    _, xd = O.quantize_rows(x[rows])
    ref = O.linear(xd, O.unpack_b(O.pack_b(W), K, N), b)
    err = O.max_rel(c.cpu().numpy()[rows], ref)
    assert err <= 1e-4, f"max-rel {err:.3e}"


@pytest.mark.parametrize("N", [3072, 384])   # the pair kernel and the 1-SM kernel
def test_linear_mirror_stores_identical_copy(env, N):
    """rl_linear_bfp16_mirror: the output and its mirror (here a second local buffer) both equal rl_linear_bfp16's
    output bit for bit, ragged M included; a mirror with fp32 output or SwiGLU is refused."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    M, K = 300, 1536
    x, W, b = _case(M, K, N, seed=12)
    _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    w = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(W)).to(dev), K, N)
    s = torch.cuda.current_stream().cuda_stream
    out = torch.full((M, N), 3.0, dtype=torch.bfloat16, device=dev)
    mir = torch.full((M, N), 5.0, dtype=torch.bfloat16, device=dev)
    L.call("rl_linear_bfp16_mirror", dq.data_ptr(), M, K, w.native.data_ptr(), N, None, L.RL_EPI_NONE, out.data_ptr(),
           mir.data_ptr(), L.RL_BF16, s)
    ref = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), N, None, L.RL_EPI_NONE, ref.data_ptr(),
           L.RL_BF16, s)
    ops.device_status()
    assert torch.equal(out, ref) and torch.equal(mir, ref)
    with pytest.raises(L.RedlineError):
        L.call("rl_linear_bfp16_mirror", dq.data_ptr(), M, K, w.native.data_ptr(), N, None, L.RL_EPI_NONE,
               out.data_ptr(), mir.data_ptr(), L.RL_F32, s)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_n_sharded_gemm_equals_unsharded_columns(env, world):
    """The N-split standalone GEMM (each GPU streams the contiguous bytes of its N / world weight columns and computes
    C[:, its columns], no collective): with whole tiles every shard's output equals the unsharded GEMM's columns bit
    for bit, at config 1's full size (X[4352, 3072] @ W[3072, 12288] + bias, bf16 out), both from the native tiles
    and from the reference's own pack_b bytes cut at rl_weights_shard's offsets; through ops.linear_bfp16 (which
    may take the split-K schedule) it agrees up to fp32 summation order and passes the oracle on sampled rows. The
    shards run one after another on one GPU: the split needs no peer, so this is the multi-GPU path's
    arithmetic."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    x, W, b = _case(4352, 3072, 12288, seed=21)
    M, K = x.shape
    N = W.shape[1]
    _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    packed = torch.from_numpy(O.pack_b(W)).to(dev)
    w = ops.PackedWeight.from_pack_b(packed, K, N)
    bt = torch.from_numpy(b).to(dev).to(torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream

    def whole_tiles(wt, bias):
        out = torch.empty((M, wt.N), dtype=torch.bfloat16, device=dev)
        L.call("rl_linear_bfp16", dq.data_ptr(), M, K, wt.native.data_ptr(), wt.N, bias.data_ptr(), L.RL_EPI_BIAS,
               out.data_ptr(), L.RL_BF16, s)
        return out
    full = whole_tiles(w, bt)
    rows = np.r_[0:8, 2040:2056, 4344:4352]
    _, xd = O.quantize_rows(x[rows])
    wd = O.unpack_b(O.pack_b(W), K, N)
    covered = 0
    for r in range(world):
        ws, n0 = w.shard(r, world)
        n1 = n0 + ws.N
        assert n0 == covered and ws.N == N // world
        covered = n1
        bs = bt[n0:n1].contiguous()
        c = whole_tiles(ws, bs)
        _, _, off, count = ops.weights_shard(K, N, r, world)
        wr = ops.PackedWeight.from_pack_b(packed[off:off + count].contiguous(), K, N // world)
        c2 = whole_tiles(wr, bs)
        csk = ops.linear_bfp16(dq, ws, bias=bs)
        ops.device_status()
        assert torch.equal(c, full[:, n0:n1]), f"shard {r}/{world} differs from the unsharded columns"
        assert torch.equal(c2, c), f"shard {r}/{world} from the reference's pack_b bytes differs"
        assert (csk.float() - c.float()).abs().max().item() <= 2.0 ** -7 * c.float().abs().max().item()
        ref = O.linear(xd, wd[:, n0:n1], b[n0:n1])
        for out in (c, csk):
            err = O.max_rel(out.float().cpu().numpy()[rows], ref)
            assert err <= BF16_OUT_TOL, f"shard {r}/{world}: max-rel {err:.3e}"
    assert covered == N


@pytest.mark.parametrize("M,N", [(4352, 3072), (300, 384), (100, 256)])
def test_linear_partial_chunk_layout(env, M, N):
    """rl_linear_bfp16_partial (the tensor-parallel projection's output): out and its mirror hold exactly
    rl_linear_bfp16's values in 16-row x 32-column chunks of 512 (chunk (r / 16, c / 32), row-major inside), ragged M
    included (the chunks wholly past M are not written, and the last chunk row's padding rows hold no data of
    interest); the pair kernel (N % 256 == 0) and the 1-SM kernel."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    K = 1536
    x, W, _ = _case(M, K, N, seed=13, bias=False)
    _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    w = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(W)).to(dev), K, N)
    s = torch.cuda.current_stream().cuda_stream
    Mp = (M + 15) // 16 * 16
    out = torch.full((Mp * N,), 3.0, dtype=torch.bfloat16, device=dev)
    mir = torch.full((Mp * N,), 5.0, dtype=torch.bfloat16, device=dev)
    L.call("rl_linear_bfp16_partial", dq.data_ptr(), M, K, w.native.data_ptr(), N, out.data_ptr(), mir.data_ptr(), s)
    ref = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), N, None, L.RL_EPI_NONE, ref.data_ptr(),
           L.RL_BF16, s)
    ops.device_status()
    for buf in (out, mir):
        rows = buf.view(Mp // 16, N // 32, 16, 32).permute(0, 2, 1, 3).reshape(Mp, N)
        assert torch.equal(rows[:M], ref)
