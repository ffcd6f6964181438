"""Generate tests/golden/golden.npz from the reference implementation itself (Cukrus-directive/redline-tiny).

Run in a container that has the reference checked out (it is never read at test time):
    python tests/golden/make_golden.py /path/to/redline-tiny
The reference's NPU runtime modules (`aie`, `aie.iron`, `aie.utils`, `pyxrt`) are replaced by empty stubs so that
its pure-numpy helpers import; nothing that needs an NPU is called. Every array below is the reference's own output
on seeded inputs (np.random.default_rng, the reference's convention), or a sha256 of it where the array is large.
"""

import hashlib
import sys
import types
from pathlib import Path

import numpy as np


def _stub_npu_modules():
    class _Any:
        def __init__(self, *a, **k):
            pass

        def __getattr__(self, name):
            return _Any()

        def __call__(self, *a, **k):
            return _Any()

    for name in ("aie", "aie.iron", "aie.utils", "aie.utils.npukernel", "aie.utils.trace", "aie.utils.trace.utils",
                 "pyxrt"):
        m = types.ModuleType(name)
        m.__getattr__ = lambda attr: _Any()
        sys.modules[name] = m
    sys.modules["aie.utils"].DefaultNPURuntime = _Any()
    sys.modules["aie.utils.npukernel"].NPUKernel = _Any


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def quant_cases(rng):
    """Edge cases for the quantiser: ties, saturation, denormals, zero blocks, wide exponent spreads."""
    blocks = []
    blocks.append(np.zeros(8, np.float32))
    blocks.append(-np.zeros(8, np.float32))
    blocks.append(np.array([1, 0, 0, 0, 0, 0, 0, 0], np.float32))
    # largest element whose scaled value is 127.5 / 127.49 / 127.51 (rounds to 128 -> saturates at 127)
    blocks.append(np.array([1.9921875, 1, 0.5, -1, -1.9921875, 0.25, 0, 3e-3], np.float32))
    blocks.append(np.array([1.99609375, -1.99609375, 0, 0, 0, 0, 0, 0], np.float32))
    blocks.append(np.array([-2 + 2 ** -7, 2 - 2 ** -8, 1, 1, 1, 1, 1, 1], np.float32))
    # ties: x * 2**(133 - E) = k + 0.5 exactly, for even and odd k
    for k in range(-6, 6):
        blocks.append(np.array([1.5, (k + 0.5) / 64, (k + 0.25) / 64, (k - 0.5) / 64, 0, 0, 0, 0], np.float32))
    # denormals and tiny values, all-denormal blocks
    d = np.array([1e-45, 2e-45, 3e-45, 1e-40, -1e-40, 1.1754942e-38, -1.17549435e-38, 5e-39], np.float32)
    blocks.append(d)
    blocks.append(np.array([1e-45, -1e-45, 0, 0, 2.8e-45, 0, 0, 0], np.float32))
    blocks.append(np.array([1e-38, 1e-45, 0, 0, 0, 0, 0, -3e-39], np.float32))
    # huge values and a wide spread inside one block
    blocks.append(np.array([3.0e38, -3.0e38, 1.0, 1e30, -1e-30, 2.0 ** 100, -2.0 ** 120, 7.0], np.float32))
    blocks.append(np.array([2.0 ** 127, 1.7e38, -1.0e38, 2.0 ** 126, 0, 0, 0, 0], np.float32))
    blocks.append(np.array([1.0, 2.0 ** -20, 2.0 ** -7, 2.0 ** -8, 2.0 ** -9, -2.0 ** -8, 3 * 2.0 ** -9, 0],
                           np.float32))
    special = np.concatenate(blocks)
    rand = np.concatenate([
        rng.standard_normal(4096).astype(np.float32),
        (rng.standard_normal(2048) * 0.02).astype(np.float32),
        (rng.standard_normal(2048) * np.exp2(rng.integers(-60, 60, 2048))).astype(np.float32),
        rng.uniform(-1, 1, 2048).astype(np.float32) * np.float32(1e-38),
    ])
    return np.concatenate([special, rand]).astype(np.float32)


def main(ref_root):
    red = Path(ref_root) / "redline"
    sys.path.insert(0, str(red))
    _stub_npu_modules()
    import npu_layouts as nl
    import pack_weights as pw
    import host_glue as hg
    import run_glue as rg
    import run_ln as rl
    import run_qkv as rq
    import forward as fw
    from ml_dtypes import bfloat16

    out = {}
    rng = np.random.default_rng(0)

    # --- a1/a2: quantiser and decoder (npu_layouts.py:62-94)
    xq = quant_cases(rng)
    out["quant_in"] = xq
    out["quant_out"] = nl.to_bfp16(xq)
    xb = rng.standard_normal(4096).astype(bfloat16).astype(np.float32)   # bf16 inputs, the GEMM activations
    out["quant_bf16_in"] = xb
    out["quant_bf16_out"] = nl.to_bfp16(xb)
    raw = rng.integers(0, 256, (512, 9), dtype=np.uint8)
    raw[:, 0] = rng.integers(0, 255, 512)                                # exponent bytes 0..254
    out["dec_in"] = raw.reshape(-1)
    out["dec_out"] = nl.from_bfp16(raw.reshape(-1)).astype(np.float64)

    # --- a3/a4/a5: layouts, as permutations of arange (npu_layouts.py:11-60)
    for name, fn, shape in (("a_layout", lambda a: nl.a_layout(a, 128, 64), (256, 128)),
                            ("b_layout", lambda a: nl.b_layout(a, 64, 128), (128, 256))):
        perm = fn(np.arange(np.prod(shape), dtype=np.int32).reshape(shape))
        out[f"{name}_{shape[0]}x{shape[1]}"] = perm.astype(np.uint16)
    perm = nl.c_layout_atb(np.arange(512 * 1024, dtype=np.int32).reshape(512, 1024), 128, 128)
    out["c_atb_512x1024_sha"] = np.frombuffer(sha(perm).encode(), np.uint8)
    pick = rng.integers(0, perm.size, 4096)
    out["c_atb_512x1024_pick"] = pick
    out["c_atb_512x1024_val"] = perm[pick]
    perm = nl.c_layout_atb(np.arange(64 * 128, dtype=np.int32).reshape(64, 128), 64, 128, rows=1, cols=1)
    out["c_atb_64x128_r1c1"] = perm.astype(np.uint16)
    # unlayouts invert the layouts (npu_layouts.py:50-60, 31-41)
    a = rng.standard_normal((256, 128)).astype(np.float32)
    out["a_unlayout_ok"] = np.array(np.array_equal(nl.a_unlayout(nl.a_layout(a, 128, 64), 256, 128, 128, 64), a))

    # --- a6: packed weights (pack_weights.py:72-89)
    W = (rng.standard_normal((128, 256)) * 0.02).astype(np.float32)      # B = W.T is (K=128, N=256)
    out["pack_in"] = W
    out["pack_out"] = pw.pack_b(W)
    wg = (rng.standard_normal((128, 64)) * 0.02).astype(np.float32)      # gate (F=128, K=64)
    wp = (rng.standard_normal((128, 64)) * 0.02).astype(np.float32)
    out["inter_gate"], out["inter_proj"] = wg, wp
    out["inter_out"] = pw.interleave_up(wg, wp)

    # --- a8: GEMM on decoded operands, float64 (the reference's check-c16 pattern, vlm_run.py:95-110)
    A = rng.standard_normal((128, 128)).astype(np.float32)
    B = (rng.standard_normal((128, 256)) * 0.02).astype(np.float32)
    ap, bp = nl.to_bfp16(nl.a_layout(A, 128, 64)), nl.to_bfp16(nl.b_layout(B, 64, 128))
    aq = nl.a_unlayout(nl.from_bfp16(ap), 128, 128, 128, 64)
    bq = nl.b_unlayout(nl.from_bfp16(bp), 128, 256, 64, 128)
    out["gemm_A"], out["gemm_B"] = A, B
    out["gemm_Apack"], out["gemm_Bpack"] = ap, bp
    out["gemm_C64"] = aq.astype(np.float64) @ bq.astype(np.float64)

    # --- a9: SwiGLU pack + reference product (run_glue.py:109-119, 141-145)
    gate = (rng.standard_normal((512, 512)) * 2).astype(np.float32)      # c_layout_atb needs M % 512, 2F % 1024
    proj = rng.standard_normal((512, 512)).astype(np.float32)
    c_pack, gq, pq = rg.swiglu_pack(gate, proj)
    out["sw_seed"] = np.array(7)
    out["sw_cpack_sha"] = np.frombuffer(sha(c_pack).encode(), np.uint8)
    ref = rg.silu(gq.astype(np.float64)) * pq
    rows = rng.integers(0, 512, 16)
    out["sw_rows"], out["sw_ref_rows"] = rows, ref[rows]
    out["sw_gate_rows"], out["sw_proj_rows"] = gate[rows], proj[rows]

    # --- a10: LN / adaLN numpy model (run_ln.py:65-71), check_random recipe at a small shape (run_ln.py:89-102)
    M, D = 256, 128
    x = rng.standard_normal((M, D)).astype(np.float32) * 3
    x[:, rng.integers(0, D, 8)] *= 40
    br = rng.standard_normal((M, D)).astype(np.float32)
    g = np.tanh(rng.standard_normal((2, D))).astype(np.float32)
    sc = (1 + 0.3 * rng.standard_normal((2, D))).astype(np.float32)
    xqln = x.astype(bfloat16).astype(np.float32)
    brq = nl.from_bfp16(nl.to_bfp16(br)).reshape(M, D)                   # row-major blocks of 8 along D
    S = 1                                                                # rows < 128 use param row 1
    gr, scr = rl.rows_param(g, M, S), rl.rows_param(sc, M, S)
    xp, y = rl.ln_ref(xqln, brq, gr, scr)
    out["ln_x"], out["ln_br"], out["ln_g"], out["ln_sc"] = xqln, brq.astype(np.float32), g, sc
    out["ln_xp"], out["ln_y"] = xp.astype(np.float32), y
    out["ln_params"] = rl.ln_params(g, sc).astype(np.float32)

    # --- a11: QK-RMSNorm + RoPE (run_glue.py:27-37) on one head of 64 tokens
    n = 64
    q = rng.standard_normal((n, 128)).astype(np.float32)
    ang = rng.uniform(-np.pi, np.pi, (n, 64))
    cos = np.cos(ang).astype(bfloat16).astype(np.float32)
    sin = np.sin(ang).astype(bfloat16).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(128)).astype(bfloat16).astype(np.float32)
    out["rr_x"], out["rr_cos"], out["rr_sin"], out["rr_w"] = q, cos, sin, w
    out["rr_out"] = rg.rms_rope(q, w, cos, sin)
    out["c_log2"] = np.array(rq.C_LOG2)

    # --- host glue: joint layout and 3-axis RoPE (host_glue.py:59-91) for the 256-text + 4096-image sequence
    pad, shapes = hg.joint_layout(np.zeros(256, bool))
    rot = hg.rope(pad, shapes)
    out["rope_t2i_shape"] = np.array(rot.shape)
    out["rope_t2i_sha"] = np.frombuffer(sha(rot).encode(), np.uint8)
    pick = rng.integers(0, rot.shape[0], 256)
    out["rope_t2i_pick"], out["rope_t2i_rows"] = pick, rot[pick]
    pad2, shapes2 = hg.joint_layout(np.array([False] * 30 + [True] * 1024 + [False] * 40))
    rot2 = hg.rope(pad2, shapes2)
    out["rope_edit_shape"] = np.array(rot2.shape)
    out["rope_edit_sha"] = np.frombuffer(sha(rot2).encode(), np.uint8)
    out["positions_8704"] = rq.positions(8704, 4128)
    # timestep embedding + modulation with small random weights (host_glue.py:31-48)
    hw = {"time_text_embed.timestep_embedder.linear_1.weight": (rng.standard_normal((64, 256)) * 0.05).astype(np.float32),
          "time_text_embed.timestep_embedder.linear_1.bias": (rng.standard_normal(64) * 0.05).astype(np.float32),
          "time_text_embed.timestep_embedder.linear_2.weight": (rng.standard_normal((64, 64)) * 0.05).astype(np.float32),
          "time_text_embed.timestep_embedder.linear_2.bias": (rng.standard_normal(64) * 0.05).astype(np.float32),
          "modulation.1.weight": (rng.standard_normal((4 * 32, 64)) * 0.05).astype(np.float32),
          "norm_out.linear.weight": (rng.standard_normal((2 * 32, 64)) * 0.05).astype(np.float32)}
    for k, v in hw.items():
        out["hw::" + k] = v
    te = hg.temb(hw, fw.model_t(0.5))
    out["temb_05"] = te
    out["mod_05"] = hg.modulation(hw, te)
    out["normout_05"] = hg.norm_out_scale(hw, te)
    out["model_t"] = np.array([fw.model_t(s) for s in fw.SIGMAS])

    # --- VAE decoder conv (vae_ops.py:44-75): the weight stream of pack_vconv and conv_ref, own seeded generator
    sys.path.insert(0, str(Path(ref_root) / "kernels" / "vae"))
    import vae_ops as vo
    rv = np.random.default_rng(11)
    wv = (rv.standard_normal((32, 16, 3, 3)) * 0.05).astype(np.float32)
    bv = (rv.standard_normal(32) * 0.01).astype(np.float32)
    xv = rv.standard_normal((6, 7, 16)).astype(np.float32)
    out["vconv_w"], out["vconv_b"], out["vconv_x"] = wv, bv, xv
    out["vconv_packed"] = vo.pack_vconv(wv, bv, 16, 16)
    out["vconv_ref"] = vo.conv_ref(xv, wv, bv)
    out["vconv1_ref"] = vo.conv_ref(xv, wv[:, :, 1:2, 1:2], bv)

    # --- the NPU attention formats (run_attn.py:29-35, 82-92) and the QKV-post table (run_qkv.py:60-72), own generator
    import run_attn as ra
    rn = np.random.default_rng(21)
    Hn, Tn = 2, 2
    qn, kn, vn = (rn.standard_normal((Hn, 64 * Tn, 128)).astype(bfloat16).astype(np.float32) for _ in range(3))
    out["npu_q"], out["npu_k"], out["npu_v"] = qn, kn, vn
    out["npu_qpack"] = np.concatenate([nl.to_bfp16(nl.a_layout(qn[h], 64, 128)) for h in range(Hn)])
    out["npu_kvpack"] = np.concatenate([ra.pack_kv(kn[h], vn[h], 64) for h in range(Hn)])
    ang = rn.uniform(-np.pi, np.pi, (64 * Tn, 64))
    cosn = np.cos(ang).astype(bfloat16).astype(np.float32)
    sinn = np.sin(ang).astype(bfloat16).astype(np.float32)
    wqn = (rn.standard_normal(128) * rq.C_LOG2).astype(bfloat16).astype(np.float32)
    wkn = (1 + 0.1 * rn.standard_normal(128)).astype(bfloat16).astype(np.float32)
    out["npu_cos"], out["npu_sin"], out["npu_wq"], out["npu_wk"] = cosn, sinn, wqn, wkn
    out["npu_tab"] = rq.qkv_tables(cosn, sinn, wqn, wkn).view(np.uint16)
    limn = rn.integers(0, 250, 64).astype(np.int32)
    out["npu_lim"], out["npu_limpack"] = limn, ra.pack_lim(limn, 64, 64)

    # --- attention: the reference's float64 causal GQA attention (vlm_run.attn_ref, vlm_run.py:181-190; 32 query
    # heads over 8 K/V heads) on bf16 inputs, own generator; inputs stored as bf16 bit patterns
    import vlm_run as vr
    ra_ = np.random.default_rng(31)
    na = 40
    qa = ra_.standard_normal((vr.HQ, na, vr.HD)).astype(bfloat16)
    ka = ra_.standard_normal((vr.HKV, na, vr.HD)).astype(bfloat16)
    va = ra_.standard_normal((vr.HKV, na, vr.HD)).astype(bfloat16)
    out["attn_q_bf16"], out["attn_k_bf16"], out["attn_v_bf16"] = (a.view(np.uint16) for a in (qa, ka, va))
    out["attn_ref"] = vr.attn_ref(qa.astype(np.float32), ka.astype(np.float32), va.astype(np.float32),
                                  na).astype(np.float32)

    dst = Path(__file__).with_name("golden.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size / 1e3:.0f} KB, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
