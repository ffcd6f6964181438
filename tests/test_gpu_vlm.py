"""GPU parity of the Qwen3-VL text-encoder path (redline_tiny_b200.vlm) against the CPU oracles:

- rl_rms_mod: x' = bf16(x + branch) bit-exact, y = RMSNorm(x') * w within max-rel 2e-2 and correlation > 0.9999
  (y is rounded to bfp16: one step is 2^-7 of a block maximum), as vlm_run.check_rms checks (vlm_run.py:73-91);
- rl_qkv_post_gqa: q / k of every head against rms_rope (max-rel 8e-3, correlation > 0.9999), V^T exact;
- rl_attention_gqa, causal: every query head against the float64 softmax over its K/V head (max-rel 2e-2,
  correlation > 0.9999, as the attention tests);
- one decoder layer (vlm.LM) against oracle/vlm_oracle.layer on the valid rows: cosine >= 0.999."""

import numpy as np
import pytest

from oracle import bfp16_oracle as O
from oracle import vlm_oracle as VO

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import ops, vlm
    assert torch.cuda.is_available()
    return torch, ops, vlm, torch.device("cuda:0")


def _bf16(torch, a, dev):
    return torch.from_numpy(O.bf16_bits(O.bf16_round(np.asarray(a, np.float32))).view(np.int16)).to(dev).view(torch.bfloat16)


def _rope(M, valid):
    pos = np.minimum(np.arange(M), valid - 1).astype(np.float64)
    inv = 1e6 ** (-np.arange(64) / 64.0)
    ang = pos[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def test_rms_mod(env):
    torch, ops, vlm, dev = env
    M, D = 512, 1024
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((M, D)) * 3).astype(np.float32)
    x[:, 7] += 40                                    # a massive-activation channel, as vlm_run.check_rms
    br = O.bf16_round(rng.standard_normal((M, D)).astype(np.float32))
    w = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    xq = O.bf16_round(x)
    xo, y, _ = ops.ln_mod(_bf16(torch, xq, dev), _bf16(torch, br, dev), vlm.rms_params(torch.from_numpy(w).to(dev)),
                          rms=True)
    ops.device_status()
    xp = O.bf16_round(xq + br)
    assert np.array_equal(xo.float().cpu().numpy(), xp)
    yr = VO.rms(xp, O.bf16_round(w))
    got = y.float().cpu().numpy()
    err, c = O.max_rel(got, yr), O.corr(got, yr)
    assert err <= 2e-2 and c > 0.9999, f"y max-rel {err:.3e} corr {c:.6f}"


@pytest.mark.parametrize("H,Hkv", [(4, 2), (8, 2), (4, 1)])
def test_qkv_post_gqa(env, H, Hkv):
    torch, ops, vlm, dev = env
    M = 320
    rng = np.random.default_rng(H * 10 + Hkv)
    qkv = O.bf16_round(rng.standard_normal((M, (H + 2 * Hkv) * 128)).astype(np.float32))
    cos, sin = _rope(M, M)
    cs = np.stack([cos, sin], -1).reshape(M, 128)
    wq = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    wk = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    q, k, vt = ops.qkv_post(_bf16(torch, qkv, dev), torch.from_numpy(cs).to(dev), torch.from_numpy(wq).to(dev),
                            torch.from_numpy(wk).to(dev), H, kv_heads=Hkv)
    ops.device_status()
    q, k, vt = (t.float().cpu().numpy() for t in (q, k, vt))
    for h in range(H):
        ref = O.rms_rope(qkv[:, h * 128:(h + 1) * 128], wq, cos, sin)
        assert O.max_rel(q[h], ref) <= 8e-3 and O.corr(q[h], ref) > 0.9999, f"q head {h}"
    for h in range(Hkv):
        ref = O.rms_rope(qkv[:, (H + h) * 128:(H + h + 1) * 128], wk, cos, sin)
        assert O.max_rel(k[h], ref) <= 8e-3 and O.corr(k[h], ref) > 0.9999, f"k head {h}"
        assert np.array_equal(vt[h][:, :M], qkv[:, (H + Hkv + h) * 128:(H + Hkv + h + 1) * 128].T), f"v head {h}"


@pytest.mark.parametrize("H,Hkv,N,valid", [(4, 2, 384, 300), (8, 2, 256, 256), (4, 1, 200, 131)])
def test_attention_gqa_causal(env, H, Hkv, N, valid):
    torch, ops, vlm, dev = env
    rng = np.random.default_rng(N)
    q = O.bf16_round(rng.standard_normal((H, N, 128)).astype(np.float32))
    k = O.bf16_round(rng.standard_normal((Hkv, N, 128)).astype(np.float32))
    v = O.bf16_round(rng.standard_normal((Hkv, N, 128)).astype(np.float32))
    ldv = (N + 127) // 128 * 128
    vt = np.zeros((Hkv, 128, ldv), np.float32)
    vt[:, :, :N] = v.transpose(0, 2, 1)
    lim = np.minimum(np.arange(N), valid - 1).astype(np.int32)
    o = ops.attention(_bf16(torch, q, dev), _bf16(torch, k, dev), _bf16(torch, vt, dev), nkv=valid,
                      row_limit=torch.from_numpy(lim).to(dev))
    ops.device_status()
    o = o.float().cpu().numpy()
    ref = VO.attention(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64), valid)
    for h in range(H):
        got = o[:, h * 128:(h + 1) * 128]
        _, refq = O.quantize_rows(ref[:, h * 128:(h + 1) * 128].astype(np.float32))
        err, c = O.max_rel(got, refq), O.corr(got, refq)
        assert err <= 2e-2 and c > 0.9999, f"head {h}: max-rel {err:.3e} corr {c:.6f}"


@pytest.mark.parametrize("dims", [dict(hidden=512, heads=4, kv_heads=2, ffn=1024, M=384, valid=300),
                                  dict(hidden=1024, heads=8, kv_heads=2, ffn=2048, M=512, valid=433)])
@pytest.mark.parametrize("fuse_qkv", [True, False])
def test_lm_layer(env, dims, fuse_qkv):
    torch, ops, vlm, dev = env
    dims = dict(dims)
    M, valid = dims.pop("M"), dims.pop("valid")
    cfg = vlm.LMConfig(**dims, layers=1)
    w = vlm.random_lm_weights(cfg, seed=7)
    lm = vlm.LM(cfg, w, M, fuse_qkv=fuse_qkv)
    cos, sin = _rope(M, valid)
    lm.set_positions(cos, sin, valid)
    rng = np.random.default_rng(7)
    x = O.bf16_round(rng.standard_normal((M, cfg.hidden)).astype(np.float32))
    lm.load_x(torch.from_numpy(x))
    lm.layer(0)
    got = lm.x_out().float().cpu().numpy()
    ops.device_status()
    lw = {k_: v_.cpu().numpy() for k_, v_ in w["layers"][0].items()}
    ref = VO.layer(x, lw, cos, sin, valid, cfg.heads, cfg.kv_heads)
    a, b = got[:valid].astype(np.float64).ravel(), ref[:valid].ravel()
    cosine = float(a @ b / np.sqrt((a @ a) * (b @ b)))
    assert cosine >= 0.999, f"layer cosine {cosine:.6f}"
