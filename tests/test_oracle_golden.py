"""Pin the CPU oracle (oracle/bfp16_oracle.py) and the host glue against the reference's own outputs
(tests/golden/golden.npz, written by tests/golden/make_golden.py from the reference's Python modules)."""

import hashlib

import numpy as np
import pytest

from oracle import bfp16_oracle as O
from oracle import host_oracle as HO
from redline_tiny_b200 import host_glue as HG


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _sha_golden(g, key):
    return bytes(g[key]).decode()


def test_to_bfp16_matches_reference_edge_cases(golden):
    got = O.to_bfp16(golden["quant_in"])
    assert np.array_equal(got, golden["quant_out"])


def test_integer_quantiser_equals_float64_quantiser(golden):
    for key in ("quant_in", "quant_bf16_in"):
        assert np.array_equal(O.to_bfp16_int(golden[key]), O.to_bfp16(golden[key]))
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(1 << 16) * np.exp2(rng.integers(-140, 120, 1 << 16))).astype(np.float32)
    assert np.array_equal(O.to_bfp16_int(x), O.to_bfp16(x))


def test_to_bfp16_bf16_inputs(golden):
    assert np.array_equal(O.to_bfp16(golden["quant_bf16_in"]), golden["quant_bf16_out"])


def test_from_bfp16(golden):
    got = O.from_bfp16(golden["dec_in"])
    assert got.dtype == np.float64
    assert np.array_equal(got, golden["dec_out"])
    # every decoded value is exact in bf16
    f32 = got.astype(np.float32)
    assert np.array_equal(O.bf16_round(f32), f32)


def test_layout_permutations(golden):
    ar = np.arange(256 * 128, dtype=np.int32).reshape(256, 128)
    assert np.array_equal(O.a_layout(ar), golden["a_layout_256x128"].astype(np.int32))
    ar = np.arange(128 * 256, dtype=np.int32).reshape(128, 256)
    assert np.array_equal(O.b_layout(ar), golden["b_layout_128x256"].astype(np.int32))
    ar = np.arange(512 * 1024, dtype=np.int32).reshape(512, 1024)
    perm = O.c_layout_atb(ar)
    assert _sha(perm) == _sha_golden(golden, "c_atb_512x1024_sha")
    ar = np.arange(64 * 128, dtype=np.int32).reshape(64, 128)
    assert np.array_equal(O.c_layout_atb(ar, 64, 128, rows=1, cols=1), golden["c_atb_64x128_r1c1"].astype(np.int32))


def test_unlayouts_invert():
    rng = np.random.default_rng(1)
    a = rng.standard_normal((256, 128)).astype(np.float32)
    assert np.array_equal(O.a_unlayout(O.a_layout(a), 256, 128), a)
    b = rng.standard_normal((128, 256)).astype(np.float32)
    assert np.array_equal(O.b_unlayout(O.b_layout(b), 128, 256), b)
    c = rng.standard_normal((512, 1024)).astype(np.float32)
    assert np.array_equal(O.c_unlayout_atb(O.c_layout_atb(c), 512, 1024), c)


def test_pack_b_and_interleave(golden):
    assert np.array_equal(O.pack_b(golden["pack_in"]), golden["pack_out"])
    assert np.array_equal(O.interleave_up(golden["inter_gate"], golden["inter_proj"]), golden["inter_out"])


def test_gemm_oracle(golden):
    A, B = golden["gemm_A"], golden["gemm_B"]
    assert np.array_equal(O.to_bfp16(O.a_layout(A)), golden["gemm_Apack"])
    assert np.array_equal(O.pack_b(B), golden["gemm_Bpack"])
    _, ad = O.quantize_rows(A)                       # row-major blocks along K == a_layout blocks
    bd = O.unpack_b(golden["gemm_Bpack"], 128, 256)
    c = O.linear(ad, bd)
    assert O.max_rel(c, golden["gemm_C64"]) < 1e-6


def test_swiglu_oracle(golden):
    rows = golden["sw_rows"]
    g, p = golden["sw_gate_rows"], golden["sw_proj_rows"]
    # swiglu_pack rounds the interleaved C through bfp16 blocks of 8 columns
    F = g.shape[1]
    c = np.empty((len(rows), 2 * F), np.float32)
    c.reshape(len(rows), F // 64, 2, 64)[:, :, 0] = g.reshape(len(rows), F // 64, 64)
    c.reshape(len(rows), F // 64, 2, 64)[:, :, 1] = p.reshape(len(rows), F // 64, 64)
    _, cq = O.quantize_rows(c)
    got = O.swiglu_from_interleaved(cq.astype(np.float64))
    assert np.allclose(got, golden["sw_ref_rows"], rtol=0, atol=1e-12)


def test_ln_ref(golden):
    M = golden["ln_x"].shape[0]
    g, sc = golden["ln_g"], golden["ln_sc"]
    gr = np.repeat(g[0:1], M, 0)
    scr = np.repeat(sc[0:1], M, 0)
    gr[:128], scr[:128] = g[1], sc[1]
    xp, y = O.ln_ref(golden["ln_x"], golden["ln_br"], gr, scr)
    assert np.array_equal(xp, golden["ln_xp"])
    assert O.max_rel(y, golden["ln_y"]) < 1e-12


def test_rms_rope(golden):
    got = O.rms_rope(golden["rr_x"], golden["rr_w"], golden["rr_cos"], golden["rr_sin"])
    assert np.allclose(got, golden["rr_out"], rtol=1e-6, atol=1e-6)
    assert float(golden["c_log2"]) == pytest.approx(np.log2(np.e) / np.sqrt(128))


def test_host_glue_rope_tables(golden):
    pad, shapes = HG.joint_layout(np.zeros(256, bool))
    rot = HG.rope(pad, shapes)
    assert list(rot.shape) == list(golden["rope_t2i_shape"]) == [4352, 64, 2]
    assert _sha(rot) == _sha_golden(golden, "rope_t2i_sha")
    pad2, shapes2 = HG.joint_layout(np.array([False] * 30 + [True] * 1024 + [False] * 40))
    rot2 = HG.rope(pad2, shapes2)
    assert list(rot2.shape) == list(golden["rope_edit_shape"])
    assert _sha(rot2) == _sha_golden(golden, "rope_edit_sha")
    assert np.array_equal(HG.positions(8704, 4128), golden["positions_8704"])


def test_host_glue_temb_modulation(golden):
    w = {k[4:]: v for k, v in golden.items() if k.startswith("hw::")}
    te = HO.temb(w, HG.model_t(0.5))
    assert np.array_equal(te, golden["temb_05"])
    assert np.array_equal(HO.modulation(w, te), golden["mod_05"])
    assert np.array_equal(HO.norm_out_scale(w, te), golden["normout_05"])
    assert np.array_equal(np.array([HG.model_t(s) for s in HG.SIGMAS]), golden["model_t"])


def test_vae_conv_oracle_and_weight_blocks(golden):
    """The VAE conv oracle reproduces vae_ops.conv_ref (3x3 and 1x1), and the B200 conv's weight rounding (pack_b
    blocks of B = [(dy, dx, ci)][co]) gives exactly the values of the reference's pack_vconv stream."""
    from oracle import vae_oracle as VO
    w, b, x = golden["vconv_w"], golden["vconv_b"], golden["vconv_x"]
    assert np.allclose(VO.conv_ref(x, w, b), golden["vconv_ref"], rtol=0, atol=1e-12)
    assert np.allclose(VO.conv_ref(x, w[:, :, 1:2, 1:2], b), golden["vconv1_ref"], rtol=0, atol=1e-12)
    ref_w = VO.unpack_vconv_weights(golden["vconv_packed"], 32, 16, 3, 16, 16)
    assert np.array_equal(VO.decode_conv_b(w), ref_w)


def test_npu_attention_formats(golden):
    """The oracle's Q / [K|V] tile packing, QKV-post table and key-limit buffer reproduce the reference's bytes
    (run_attn.pack_kv / a_layout Q tiles, run_qkv.qkv_tables, run_attn.pack_lim)."""
    from oracle import npu_oracle as N
    q, k, v = golden["npu_q"], golden["npu_k"], golden["npu_v"]
    assert np.array_equal(N.q_pack(q), golden["npu_qpack"])
    assert np.array_equal(N.kv_pack(k, v), golden["npu_kvpack"])
    # decoding gives each value's bfp16 rounding (re-encoding is not byte-identical: a block whose negative maximum
    # rounds to -128 decodes to -2^(E - 126), which encodes with exponent E + 1)
    qd = N.q_unpack(golden["npu_qpack"], 2)
    kd, vd = N.kv_unpack(golden["npu_kvpack"], 2)
    for got, ref in ((qd, q), (kd, k), (vd, v)):
        assert np.abs(got - ref).max() <= 2.0 ** -6 * np.abs(ref).max()
    tab = N.tables(golden["npu_cos"], golden["npu_sin"], golden["npu_wq"], golden["npu_wk"])
    assert np.array_equal(tab, golden["npu_tab"])
    cos, sin, wq, wk = N.tables_decode(golden["npu_tab"])
    for got, name in ((cos, "npu_cos"), (sin, "npu_sin"), (wq, "npu_wq"), (wk, "npu_wk")):
        assert np.array_equal(got, golden[name]), name
    assert np.array_equal(N.lim_pack(golden["npu_lim"]), golden["npu_limpack"])


def attn_golden_inputs(g):
    """The golden attention case as float32 arrays: q (32, n, 128), k / v (8, n, 128), all bf16 values."""
    return tuple(O.bf16_from_bits(g[k]).astype(np.float32) for k in ("attn_q_bf16", "attn_k_bf16", "attn_v_bf16"))


def test_attention_oracle_matches_reference_attn_ref(golden):
    """oracle.attention_f64 (the float64 softmax used by every attention parity test) against the reference's own
    float64 causal GQA attention, vlm_run.attn_ref (redline/vlm_run.py:181-190): query head h reads K/V head h // 4
    and row r sees keys <= r (the per-row key limit form, run_attn.py:123-126)."""
    q, k, v = attn_golden_inputs(golden)
    H, n, _ = q.shape
    ref = golden["attn_ref"]
    assert ref.shape == (n, H * 128)
    for h in range(H):
        got = O.attention_f64(q[h], k[h // (H // k.shape[0])], v[h // (H // k.shape[0])], row_limit=np.arange(n))
        assert np.allclose(got, ref[:, h * 128:(h + 1) * 128], rtol=1e-6, atol=1e-7), f"head {h}"
