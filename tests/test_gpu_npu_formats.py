"""The NPU attention formats on the GPU (rl_npu_*) and the drop-in Device's QKV-post and attention artifacts, driven
with buffers in the reference's formats: Q / [K|V] tiles, the QKV-post table and the key-limit buffer made by the
oracle (oracle/npu_oracle.py, pinned against the reference's run_attn.pack_kv / run_qkv.qkv_tables / pack_lim bytes
in tests/golden), O read back with a_unlayout.

Tolerances: packing bf16 values is bit-exact against the reference's bytes; the QKV post matches the float64
RMSNorm / RoPE oracle within two bfp16 steps (its values pass through bf16 before the bfp16 packing), and attention
(P in bf16, O in bfp16) within max-rel 2e-2 with correlation > 0.9999, as tests/test_gpu_attention.py."""

import math

import numpy as np
import pytest

from oracle import bfp16_oracle as O
from oracle import npu_oracle as N

pytestmark = pytest.mark.gpu
LN2 = math.log(2.0)


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import _lib as L
    from redline_tiny_b200 import npu
    assert torch.cuda.is_available()
    return torch, L, npu, torch.device("cuda:0")


def _bf16(torch, a, dev):
    return torch.from_numpy(O.bf16_bits(O.bf16_round(np.asarray(a, np.float32))).view(np.int16)).to(dev).view(
        torch.bfloat16)


def _u8(torch, a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint8)).to(dev)


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def test_pack_matches_reference_bytes(env, golden):
    torch, L, _, dev = env
    q, k, v = golden["npu_q"], golden["npu_k"], golden["npu_v"]
    H, M = q.shape[0], q.shape[1]
    qd, kd = _bf16(torch, q, dev), _bf16(torch, k, dev)
    vt = _bf16(torch, np.ascontiguousarray(v.transpose(0, 2, 1)), dev)
    qo = torch.empty(golden["npu_qpack"].size, dtype=torch.uint8, device=dev)
    kvo = torch.empty(golden["npu_kvpack"].size, dtype=torch.uint8, device=dev)
    L.call("rl_npu_qkv_pack", qd.data_ptr(), kd.data_ptr(), vt.data_ptr(), M, H, M // 64, qo.data_ptr(),
           kvo.data_ptr(), _stream(torch))
    assert np.array_equal(qo.cpu().numpy(), golden["npu_qpack"])
    assert np.array_equal(kvo.cpu().numpy(), golden["npu_kvpack"])


def test_unpack_tile_ranges(env, golden):
    """Q tiles and K/V tile ranges decoded at key offsets equal the oracle's decoding."""
    torch, L, _, dev = env
    H = 2
    qb, kvb = _u8(torch, golden["npu_qpack"], dev), _u8(torch, golden["npu_kvpack"], dev)
    qref = N.q_unpack(golden["npu_qpack"], H)
    kref, vref = N.kv_unpack(golden["npu_kvpack"], H)
    q = torch.empty(H, 64, 128, dtype=torch.bfloat16, device=dev)
    L.call("rl_npu_q_unpack", qb.data_ptr(), H, 2, 1, 1, q.data_ptr(), _stream(torch))     # tile 1 of 2
    assert np.array_equal(q.float().cpu().numpy(), qref[:, 64:128])
    nk = 192
    k = torch.zeros(H, nk, 128, dtype=torch.bfloat16, device=dev)
    vt = torch.zeros(H, 128, nk, dtype=torch.bfloat16, device=dev)
    L.call("rl_npu_kv_unpack", kvb.data_ptr(), H, 2, 0, 2, 64, nk, nk, k.data_ptr(), vt.data_ptr(), _stream(torch))
    assert np.array_equal(k.float().cpu().numpy()[:, 64:], kref)
    assert np.array_equal(vt.float().cpu().numpy()[:, :, 64:], vref.transpose(0, 2, 1))
    assert not k.float().cpu().numpy()[:, :64].any()
    with pytest.raises(L.RedlineError):      # tile range outside the buffer: refused before any launch
        L.call("rl_npu_kv_unpack", kvb.data_ptr(), H, 2, 1, 2, 0, nk, nk, k.data_ptr(), vt.data_ptr(), 0)


def test_tables_decode(env, golden):
    torch, L, _, dev = env
    tab = torch.from_numpy(golden["npu_tab"].view(np.int16)).to(dev)
    T = golden["npu_tab"].shape[0]
    cs = torch.empty(64 * T, 64, 2, dtype=torch.float32, device=dev)
    wq = torch.empty(128, dtype=torch.float32, device=dev)
    wk = torch.empty(128, dtype=torch.float32, device=dev)
    L.call("rl_npu_qkv_tables", tab.data_ptr(), T, cs.data_ptr(), wq.data_ptr(), wk.data_ptr(), _stream(torch))
    c = cs.cpu().numpy()
    assert np.array_equal(c[..., 0], golden["npu_cos"]) and np.array_equal(c[..., 1], golden["npu_sin"])
    assert np.array_equal(wq.cpu().numpy(), golden["npu_wq"]) and np.array_equal(wk.cpu().numpy(), golden["npu_wk"])


def test_device_qkv_post(env):
    """npu.run("qkv_post", QKV_ART[M], [C_qkv, tabs, Q, KV]) (forward.py:246) against RMSNorm * w + RoPE in float64
    on the bfp16-decoded C, packed by the oracle."""
    torch, L, npu, dev = env
    M, H = 512, 8
    HID = 128 * H
    rng = np.random.default_rng(5)
    C = rng.standard_normal((M, 3 * HID)).astype(np.float32)
    ang = rng.uniform(-np.pi, np.pi, (M, 64))
    cos, sin = O.bf16_round(np.cos(ang).astype(np.float32)), O.bf16_round(np.sin(ang).astype(np.float32))
    wq = O.bf16_round((rng.standard_normal(128) * np.log2(np.e) / np.sqrt(128)).astype(np.float32))
    wk = O.bf16_round((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))
    cq = O.to_bfp16(O.c_layout_atb(C))
    tab = N.tables(cos, sin, wq, wk)
    T = M // 64
    qb = torch.zeros(H * T * 9216, dtype=torch.uint8, device=dev)
    kvb = torch.zeros(2 * H * T * 9216, dtype=torch.uint8, device=dev)
    d = npu.Device()
    d.run("qkv_post", f"glue-qkv32-m{M}", [_u8(torch, cq, dev), torch.from_numpy(tab.view(np.int16)).to(dev), qb, kvb])
    d.sync()
    qg = N.q_unpack(qb.cpu().numpy(), H)
    kg, vg = N.kv_unpack(kvb.cpu().numpy(), H)
    Cd = O.c_unlayout_atb(O.from_bfp16(cq), M, 3 * HID)
    for h in range(H):
        qr = O.rms_rope(Cd[:, h * 128:(h + 1) * 128], wq, cos, sin)
        kr = O.rms_rope(Cd[:, HID + h * 128:HID + (h + 1) * 128], wk, cos, sin)
        vr = Cd[:, 2 * HID + h * 128:2 * HID + (h + 1) * 128]
        for got, ref, name in ((qg[h], qr, "q"), (kg[h], kr, "k"), (vg[h], vr, "v")):
            err = np.abs(got - ref).max() / np.abs(ref).max()
            assert err <= 2 * 2.0 ** -7 and O.corr(got, ref) > 0.9999, f"head {h} {name}: max-rel {err:.3e}"


def _attn_ref(q, k, v, nkv, lim=None):
    """Softmax in float64 of q . k (q carries log2(e) / sqrt(128): logits in log2 units) over the first nkv keys."""
    s = (q.astype(np.float64) @ k[:nkv].astype(np.float64).T) * LN2
    if lim is not None:
        s = np.where(np.arange(nkv)[None, :] <= np.asarray(lim)[:, None], s, -np.inf)
    w = np.exp(s - s.max(1, keepdims=True))
    return (w / w.sum(1, keepdims=True)) @ v[:nkv].astype(np.float64)


def _check_o(ob, rows, H, nq, refs):
    o = O.a_unlayout(O.from_bfp16(ob), rows, H * 128)
    for h, ref in enumerate(refs):
        _, refq = O.quantize_rows(ref.astype(np.float32))
        got = o[:nq, h * 128:(h + 1) * 128]
        err, c = O.max_rel(got, refq), O.corr(got, refq)
        assert err <= 2e-2 and c > 0.9999, f"head {h}: max-rel {err:.3e} corr {c:.6f}"
    return o


def _rand_qkv(rng, H, n):
    q = O.bf16_round((rng.standard_normal((H, n, 128)) * 0.12).astype(np.float32))
    k = O.bf16_round(rng.standard_normal((H, n, 128)).astype(np.float32))
    v = O.bf16_round(rng.standard_normal((H, n, 128)).astype(np.float32))
    return q, k, v


def test_device_attention_cached_step(env):
    """attn32o ... -s- ... -pf- (forward.py:613, CachedStep.blocks): every Q tile over [target K/V | prefix tiles]."""
    torch, L, npu, dev = env
    rng = np.random.default_rng(6)
    H, Tq, Tp, npre = 2, 2, 5, 3
    q, kt, vt_ = _rand_qkv(rng, H, 64 * Tq)
    _, kp, vp = _rand_qkv(rng, H, 64 * Tp)
    NK, NKV = 64 * (Tq + npre), 64 * (Tq + npre) - 20
    qb = N.q_pack(q)
    qd = N.q_unpack(qb, H)
    kvt, kvp = N.kv_pack(kt, vt_), N.kv_pack(kp, vp)
    ktd, vtd = N.kv_unpack(kvt, H)
    kpd, vpd = N.kv_unpack(kvp, H)
    ob = torch.zeros(128 * H * 128 // 8 * 9, dtype=torch.uint8, device=dev)
    d = npu.Device()
    d.run("attn", f"attn32o-v6-s-h{H}-t8-pf-nk{NK}-nkv{NKV}", [_u8(torch, qb, dev), _u8(torch, kvt, dev),
                                                                _u8(torch, kvp, dev), ob])
    d.sync()
    refs = []
    for h in range(H):
        kk = np.concatenate([ktd[h], kpd[h, :64 * npre]])
        vv = np.concatenate([vtd[h], vpd[h, :64 * npre]])
        refs.append(_attn_ref(qd[h], kk, vv, NKV))
    _check_o(ob.cpu().numpy(), 128, H, 64 * Tq, refs)


def test_device_attention_reference_rows(env):
    """attn32o ... -a- ... -tr- (ExtractStep.blocks): Q tiles 0.. over K/V tiles 0.. of one buffer."""
    torch, L, npu, dev = env
    rng = np.random.default_rng(7)
    H, T = 2, 4
    q, k, v = _rand_qkv(rng, H, 64 * T)
    qb, kv = N.q_pack(q), N.kv_pack(k, v)
    qd = N.q_unpack(qb, H)
    kd, vd = N.kv_unpack(kv, H)
    NK, NKV = 192, 180
    ob = torch.zeros(256 * H * 128 // 8 * 9, dtype=torch.uint8, device=dev)
    d = npu.Device()
    d.run("attn_ref", f"attn32o-v6-a-h{H}-t8-tr-nk{NK}-nkv{NKV}", [_u8(torch, qb, dev), _u8(torch, kv, dev), ob])
    d.sync()
    _check_o(ob.cpu().numpy(), 256, H, 256, [_attn_ref(qd[h], kd[h], vd[h], NKV) for h in range(H)])


def test_device_attention_step1_target(env):
    """attn32o ... -s- ... -tr- (ExtractStep.blocks at the text-to-image layout M = 4608, target from row 512):
    Q / K / V tiles 8..71 over [those | prefix tiles 0..1] of the same full buffer."""
    torch, L, npu, dev = env
    rng = np.random.default_rng(8)
    H, T = 1, 72
    q, k, v = _rand_qkv(rng, H, 64 * T)
    qb, kv = N.q_pack(q), N.kv_pack(k, v)
    qd = N.q_unpack(qb, H)
    kd, vd = N.kv_unpack(kv, H)
    NK, NKV = 4096 + 128, 4096 + 100
    kvd = _u8(torch, kv, dev)
    ob = torch.zeros(4096 * H * 128 // 8 * 9, dtype=torch.uint8, device=dev)
    d = npu.Device()
    d.run("attn", f"attn32o-v6-s-h{H}-t8-tr-nk{NK}-nkv{NKV}", [_u8(torch, qb, dev), kvd, kvd, ob])
    d.sync()
    kk = np.concatenate([kd[0, 512:512 + 4096], kd[0, :128]])
    vv = np.concatenate([vd[0, 512:512 + 4096], vd[0, :128]])
    _check_o(ob.cpu().numpy(), 4096, H, 4096, [_attn_ref(qd[0, 512:512 + 4096], kk, vv, NKV)])


def test_device_attention_small_query_limits(env):
    """attn32q (ExtractStep host rows): 32 heads x 64 queries over K/V tiles 0.. of a [head][PT] buffer with per-row
    key limits from the LIM buffer (run_attn.pack_lim)."""
    torch, L, npu, dev = env
    rng = np.random.default_rng(9)
    H, PT, NK = 32, 3, 128
    q, _, _ = _rand_qkv(rng, H, 64)
    _, k, v = _rand_qkv(rng, H, 64 * PT)
    lim = rng.integers(0, NK - 1, 64).astype(np.int32)
    lim[:6] = np.arange(6)
    qb, kv = N.q_pack(q), N.kv_pack(k, v)
    qd = N.q_unpack(qb, H)
    kd, vd = N.kv_unpack(kv, H)
    ob = torch.zeros(128 * H * 128 // 8 * 9, dtype=torch.uint8, device=dev)
    d = npu.Device()
    d.run("attn_small", f"attn32q-v6-t8-nk{NK}-pt{PT}", [_u8(torch, qb, dev), _u8(torch, N.lim_pack(lim), dev),
                                                        _u8(torch, kv, dev), ob])
    d.sync()
    o = _check_o(ob.cpu().numpy(), 128, H, 64, [_attn_ref(qd[h], kd[h], vd[h], NK, lim) for h in range(H)])
    assert not o[64:].any()


def test_device_rejects_unknown_attention_form(env):
    torch, L, npu, dev = env
    with pytest.raises(NotImplementedError):
        npu.Device().run("attn", "attn32x-unknown", [])
