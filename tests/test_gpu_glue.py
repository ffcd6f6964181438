"""GPU parity of the SwiGLU MLP entry (config 2), the adaLN residual + LayerNorm kernel and the QK-RMSNorm + RoPE
kernel against the CPU oracle (oracle/bfp16_oracle.py: the reference's numpy models run_ln.ln_ref,
run_glue.rms_rope and the decoded-operand float32 GEMMs).

Tolerances: x' of ln_mod is bit-exact (the reference reports it bit-exact, run_ln.py:106-107); y = LN(x') * sc is
rounded to bfp16, so it is compared with max-rel <= 2e-2 (one bfp16 step is 2^-7 of a block's largest value) and
correlation > 0.9999 (run_ln.py:112); RMSNorm + RoPE outputs are bf16, max-rel <= 8e-3 and correlation > 0.9999
(run_qkv.py:148 asks > 0.999); the MLP output (fp32) max-rel <= 2e-3 against the fp32 oracle - its H is rounded to
bfp16 on both sides, so the rare rounding tie that goes the other way moves one H value by one bfp16 step."""

import numpy as np
import pytest

from oracle import bfp16_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import ops
    assert torch.cuda.is_available()
    return torch, ops, torch.device("cuda:0")


def _bf16(torch, a, dev):
    return torch.from_numpy(O.bf16_bits(O.bf16_round(a)).view(np.int16)).to(dev).view(torch.bfloat16)


def _mlp_case(M, K, F, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wg = (rng.standard_normal((F, K)) * 0.02).astype(np.float32)
    wu = (rng.standard_normal((F, K)) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((N, F)) * 0.02).astype(np.float32)
    return x, O.interleave_up(wg, wu), wd.T.copy()


def _mlp_oracle(x, Bup, Bdown):
    _, xd = O.quantize_rows(x)
    K, F2 = Bup.shape
    c = O.linear(xd, O.unpack_b(O.pack_b(Bup), K, F2))
    _, h = O.quantize_rows(O.swiglu_from_interleaved(c))
    F, N = Bdown.shape
    return O.linear(h, O.unpack_b(O.pack_b(Bdown), F, N))


@pytest.mark.parametrize("M,K,F,N", [(128, 256, 256, 128), (300, 512, 384, 256), (512, 4096, 12288, 4096)])
def test_swiglu_mlp(env, M, K, F, N):
    """Config 2 (Qwen3-VL SwiGLU MLP, X[512, 4096], gate/up [4096, 12288], down [12288, 4096]) and smaller cases."""
    torch, ops, dev = env
    x, Bup, Bdown = _mlp_case(M, K, F, N, seed=M + K)
    wu = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(Bup)).to(dev), K, 2 * F, swiglu=True)
    wd = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(Bdown)).to(dev), F, N)
    out = ops.swiglu_mlp(_bf16(torch, x, dev), wu, wd, out_dtype=torch.float32)
    ops.device_status()
    ref = _mlp_oracle(O.bf16_round(x), Bup, Bdown)
    got = out.float().cpu().numpy()
    err = O.max_rel(got, ref)
    assert err <= 2e-3, f"max-rel {err:.3e} corr {O.corr(got, ref):.6f}"


def test_swiglu_mlp_prequantized_and_workspace(env):
    torch, ops, dev = env
    M, K, F, N = 256, 256, 256, 256
    x, Bup, Bdown = _mlp_case(M, K, F, N, seed=9)
    wu = ops.PackedWeight.from_float(torch.from_numpy(Bup).to(dev), swiglu=True)
    wd = ops.PackedWeight.from_float(torch.from_numpy(Bdown).to(dev))
    _, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    a = ops.swiglu_mlp(dq, wu, wd, x_quantized=True, out_dtype=torch.float32)
    b = ops.swiglu_mlp(torch.from_numpy(x).to(dev), wu, wd, out_dtype=torch.float32)
    assert torch.equal(a, b)
    from redline_tiny_b200 import _lib as L
    small = torch.empty(16, dtype=torch.uint8, device=dev)
    with pytest.raises(L.RedlineError):
        ops.swiglu_mlp(dq, wu, wd, x_quantized=True, workspace=small)


def _ln_inputs(M, D, seed):
    """run_ln.check_random's recipe (run_ln.py:91-96): x*3 with outlier channels, a bfp16 branch, g = tanh, sc = 1 +
    0.3 N(0,1), two parameter rows."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, D)).astype(np.float32) * 3
    x[:, rng.integers(0, D, 8)] *= 40
    br = rng.standard_normal((M, D)).astype(np.float32)
    g = np.tanh(rng.standard_normal((2, D))).astype(np.float32)
    sc = (1 + 0.3 * rng.standard_normal((2, D))).astype(np.float32)
    return O.bf16_round(x), O.quantize_rows(br)[1], g, sc


@pytest.mark.parametrize("M,D,split", [(256, 128, 128), (300, 3072, 0), (4352, 3072, 256), (100, 1032, 50),
                                     (200, 4096, 0), (64, 8256, 10)])
def test_ln_mod(env, golden, M, D, split):
    torch, ops, dev = env
    if M == 256 and D == 128:
        x, br, g, sc = golden["ln_x"], golden["ln_br"], golden["ln_g"], golden["ln_sc"]
    else:
        x, br, g, sc = _ln_inputs(M, D, seed=M)
    params = O.bf16_round(np.concatenate([g, sc], 1).reshape(2, 2, D))
    xo, y, yq = ops.ln_mod(_bf16(torch, x, dev), _bf16(torch, br, dev), _bf16(torch, params, dev), row_split=split,
                           want_y_bytes=True)
    ops.device_status()
    gr = np.repeat(g[0:1], M, 0)
    scr = np.repeat(sc[0:1], M, 0)
    gr[:split], scr[:split] = g[1], sc[1]
    xp_ref, y_ref = O.ln_ref(x, br, gr, scr)
    got_x = xo.float().cpu().numpy()
    assert np.array_equal(got_x, xp_ref), f"x' differs in {np.sum(got_x != xp_ref)} of {got_x.size}"
    got_y = y.float().cpu().numpy()
    err = O.max_rel(got_y, y_ref)
    c = O.corr(got_y, y_ref)
    assert err <= 2e-2 and c > 0.9999, f"y max-rel {err:.3e} corr {c:.6f}"
    # the bytes decode to the same values, and equal the oracle's quantisation of our own y in >= 99% of blocks
    assert np.array_equal(O.from_bfp16(yq.cpu().numpy()).astype(np.float32).reshape(M, D), got_y)
    if M == 256:
        assert np.array_equal(xp_ref, golden["ln_xp"])


def test_ln_mod_no_branch(env):
    torch, ops, dev = env
    M, D = 128, 256
    x, _, g, sc = _ln_inputs(M, D, seed=3)
    params = O.bf16_round(np.concatenate([g, sc], 1).reshape(2, 2, D))
    xo, y, _ = ops.ln_mod(_bf16(torch, x, dev), None, _bf16(torch, params, dev))
    xp_ref, y_ref = O.ln_ref(x, np.zeros_like(x), np.repeat(g[:1], M, 0), np.repeat(sc[:1], M, 0))
    assert np.array_equal(xo.float().cpu().numpy(), x)
    assert O.max_rel(y.float().cpu().numpy(), y_ref) <= 2e-2


@pytest.mark.parametrize("M,H", [(64, 1), (300, 3), (4352, 24)])
def test_qkv_post(env, golden, M, H):
    torch, ops, dev = env
    rng = np.random.default_rng(M + H)
    qkv = O.bf16_round(rng.standard_normal((M, 3 * H * 128)).astype(np.float32))
    ang = rng.uniform(-np.pi, np.pi, (M, 64))
    cs = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    wq = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32) * np.float32(np.log2(np.e) / np.sqrt(128))
    wk = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    ldv = (M + 127) // 128 * 128
    q, k, vt = ops.qkv_post(_bf16(torch, qkv, dev), torch.from_numpy(cs).to(dev), torch.from_numpy(wq).to(dev),
                            torch.from_numpy(wk).to(dev), H, ldv=ldv)
    ops.device_status()
    q, k, vt = (t.float().cpu().numpy() for t in (q, k, vt))
    for h in range(H):
        qr = O.rms_rope(qkv[:, h * 128:(h + 1) * 128], wq, cs[..., 0], cs[..., 1])
        kr = O.rms_rope(qkv[:, (H + h) * 128:(H + h + 1) * 128], wk, cs[..., 0], cs[..., 1])
        for got, ref in ((q[h], qr), (k[h], kr)):
            err, c = O.max_rel(got, ref), O.corr(got, ref)
            assert err <= 8e-3 and c > 0.9999, f"head {h}: max-rel {err:.3e} corr {c:.6f}"
        v = qkv[:, (2 * H + h) * 128:(2 * H + h + 1) * 128]
        assert np.array_equal(vt[h][:, :M], v.T)
        assert not vt[h][:, M:].any()


@pytest.mark.parametrize("M,K,H,Hkv,ldv", [(300, 256, 2, 2, None), (300, 512, 4, 1, 304), (200, 512, 4, 1, 256),
                                           (1088, 2048, 32, 8, None), (4352, 3072, 24, 24, None),
                                           (300, 256, 1, 1, None), (4352, 3072, 3, 3, None)])
def test_qkv_linear_fused(env, M, K, H, Hkv, ldv):
    """rl_qkv_linear (QK-RMSNorm + RoPE in the QKV GEMM's epilogue) against the two-launch form it replaces:
    rl_linear_bfp16 (the same kernel - the 2-SM pair kernel for an even head count, the 1-SM one for an odd count -
    so the same fp32 accumulators) followed by rl_qkv_post_gqa. V is the same
    bf16 rounding of the same accumulator: bit-exact, zero columns M..ldv-1 included. q / k sum their squares in
    another order and may contract the RoPE products into FMAs differently, so a value may land one bf16 step away:
    >= 97% bit-identical, and within 2^-6 of the head's largest |value|; both forms meet the oracle's rms_rope bar
    of test_qkv_post."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    rng = np.random.default_rng(M + 7 * H + Hkv)
    N = (H + 2 * Hkv) * 128
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(dev)
    _, xdq = ops.quantize_bfp16(x.to(torch.bfloat16), want_bytes=False)
    W = torch.from_numpy((rng.standard_normal((K, N)) * 0.03).astype(np.float32)).to(dev)
    w = ops.PackedWeight.from_float(W)
    ang = rng.uniform(-np.pi, np.pi, (M, 64))
    cs = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    wq = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32) * np.float32(np.log2(np.e) / np.sqrt(128))
    wk = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    cs_t, wq_t, wk_t = (torch.from_numpy(a).to(dev) for a in (cs, wq, wk))
    qkv = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    L.call("rl_linear_bfp16", xdq.data_ptr(), M, K, w.native.data_ptr(), N, None, L.RL_EPI_NONE, qkv.data_ptr(),
           L.RL_BF16, torch.cuda.current_stream().cuda_stream)
    q0, k0, vt0 = ops.qkv_post(qkv, cs_t, wq_t, wk_t, H, ldv=ldv, kv_heads=Hkv)
    vt1 = torch.full_like(vt0, 7.0)           # the fused form must write the padding columns too
    q1, k1, _ = ops.qkv_linear(xdq, w, cs_t, wq_t, wk_t, H, ldv=ldv, kv_heads=Hkv)
    L.call("rl_qkv_linear", xdq.data_ptr(), M, K, w.native.data_ptr(), H, Hkv, cs_t.data_ptr(), wq_t.data_ptr(),
           wk_t.data_ptr(), q1.data_ptr(), k1.data_ptr(), vt1.data_ptr(), vt0.shape[2],
           torch.cuda.current_stream().cuda_stream)
    ops.device_status()
    assert torch.equal(vt1.view(torch.int16), vt0.view(torch.int16))
    qkv_np = qkv.float().cpu().numpy()
    for name, a, b in (("q", q1, q0), ("k", k1, k0)):
        same = (a.view(torch.int16) == b.view(torch.int16)).float().mean().item()
        assert same >= 0.97, f"{name}: only {same:.4f} of values bit-identical"
        for hh in range(a.shape[0]):
            lim = 2.0 ** -6 * b[hh].float().abs().max().item()
            d = (a[hh].float() - b[hh].float()).abs().max().item()
            assert d <= lim, f"{name} head {hh}: max |fused - unfused| {d:.3e} > {lim:.3e}"
    q1n, k1n = q1.float().cpu().numpy(), k1.float().cpu().numpy()
    for hh in range(min(H, 4)):
        ref = O.rms_rope(qkv_np[:, hh * 128:(hh + 1) * 128], wq, cs[..., 0], cs[..., 1])
        err, c = O.max_rel(q1n[hh], ref), O.corr(q1n[hh], ref)
        assert err <= 8e-3 and c > 0.9999, f"q head {hh}: max-rel {err:.3e} corr {c:.6f}"
    for hh in range(min(Hkv, 4)):
        ref = O.rms_rope(qkv_np[:, (H + hh) * 128:(H + hh + 1) * 128], wk, cs[..., 0], cs[..., 1])
        err, c = O.max_rel(k1n[hh], ref), O.corr(k1n[hh], ref)
        assert err <= 8e-3 and c > 0.9999, f"k head {hh}: max-rel {err:.3e} corr {c:.6f}"


def test_qkv_linear_rejects_bad_shapes(env):
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    x = torch.zeros(64, 128, dtype=torch.bfloat16, device=dev)
    cs = torch.zeros(64, 64, 2, device=dev)
    wn = torch.ones(128, device=dev)
    w3 = ops.PackedWeight.from_float(torch.zeros(128, 3 * 128, device=dev))
    with pytest.raises(L.RedlineError):
        ops.qkv_linear(torch.zeros(64, 96, dtype=torch.bfloat16, device=dev), w3, cs, wn, wn, 1)   # K % 64 != 0
    w4 = ops.PackedWeight.from_float(torch.zeros(128, 4 * 128, device=dev))   # H 2, Hkv 1
    with pytest.raises(ValueError):
        ops.qkv_linear(x, w4, cs, wn, wn, 2)                                  # Hkv 2 would need 6 heads
    with pytest.raises(L.RedlineError):
        ops.qkv_linear(x, w4, cs, wn, wn, 2, kv_heads=1, ldv=72)              # ldv % 16 != 0
    with pytest.raises(L.RedlineError):
        ops.qkv_linear(x, w4, cs, wn, wn, 2, kv_heads=1, ldv=512)             # past M rounded up to 256
    ops.device_status()
