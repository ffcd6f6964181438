"""The drop-in Device (redline_tiny_b200.npu) driven exactly as the reference drives its NPU: buffers in the
reference's formats built by the oracle (to_bfp16(a_layout(.)), pack_b, c_layout_atb, ln_params), results read
back with the reference's own unlayouts, compared with the oracle on the same inputs. The C-order bytes of the
quantiser are also checked bit-exact against to_bfp16(c_layout_atb(.)).

Tolerances: outputs are bfp16 (one step is 2^-7 of a block maximum), so max-rel <= 2e-2 with correlation > 0.9999;
x' of ln_mod is bit-exact."""

import numpy as np
import pytest

from oracle import bfp16_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import npu, ops
    return torch, npu, ops, torch.device("cuda:0")


def _u8(torch, a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint8)).to(dev)


def _bf16(torch, a, dev):
    return torch.from_numpy(O.bf16_bits(O.bf16_round(a)).view(np.int16)).to(dev).view(torch.bfloat16)


def test_c_order_quantiser_and_permutation_bit_exact(env):
    torch, npu, ops, dev = env
    M, N = 1024, 2048
    x = O.bf16_round(np.random.default_rng(0).standard_normal((M, N)).astype(np.float32))
    q, _ = ops.quantize_bfp16(_bf16(torch, x, dev), layout="c_atb")
    assert np.array_equal(q.cpu().numpy(), O.to_bfp16(O.c_layout_atb(x)))
    p = ops.permute_bf16(_bf16(torch, x, dev).reshape(-1), M, N, src="rowmajor", dst="c_atb")
    assert np.array_equal(p.float().cpu().numpy(), O.c_layout_atb(x))
    back = ops.permute_bf16(p, M, N, src="c_atb", dst="a_layout")
    assert np.array_equal(back.float().cpu().numpy(), O.a_layout(x))
    d = ops.dequantize_bfp16(q, M, N, layout="c_atb")
    assert np.array_equal(d.cpu().numpy(), O.quantize_rows(x)[1])


def test_device_gemm(env):
    """gemm(npu, w, op, M, a, c) (forward.py:194-197): A = to_bfp16(a_layout(X)), B = pack_b(W), C in ATB order."""
    torch, npu, ops, dev = env
    M, K, N = 512, 256, 1024
    rng = np.random.default_rng(1)
    X = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    A, B = O.to_bfp16(O.a_layout(X)), O.pack_b(W)
    C = torch.zeros(M * N // 8 * 9, dtype=torch.uint8, device=dev)
    d = npu.Device()
    d.run("qkv", "atb3d2-qkv", [_u8(torch, A, dev), _u8(torch, B, dev), C])
    d.sync()
    got = O.c_unlayout_atb(O.from_bfp16(C.cpu().numpy()).astype(np.float32), M, N)
    ref = O.linear(O.a_unlayout(O.from_bfp16(A).astype(np.float32), M, K), O.unpack_b(B, K, N))
    err, c = O.max_rel(got, ref), O.corr(got, ref)
    assert err <= 2e-2 and c > 0.9999, f"max-rel {err:.3e} corr {c:.6f}"
    same = np.mean(C.cpu().numpy().reshape(-1, 9) == O.to_bfp16(O.c_layout_atb(ref)).reshape(-1, 9))
    assert same > 0.99


def test_device_up_swiglu(env):
    """npu.run("up_swiglu", ...) (forward.py:250): H = silu(gate) * proj as the down GEMM's a_layout A operand."""
    torch, npu, ops, dev = env
    M, K, F = 256, 256, 512
    rng = np.random.default_rng(2)
    X = rng.standard_normal((M, K)).astype(np.float32)
    Bup = O.interleave_up((rng.standard_normal((F, K)) * 0.02).astype(np.float32),
                          (rng.standard_normal((F, K)) * 0.02).astype(np.float32))
    A, B = O.to_bfp16(O.a_layout(X)), O.pack_b(Bup)
    H = torch.zeros(M * F // 8 * 9, dtype=torch.uint8, device=dev)
    npu.Device().run("up_swiglu", "atb3sw2-m256", [_u8(torch, A, dev), _u8(torch, B, dev), H])
    got = O.a_unlayout(O.from_bfp16(H.cpu().numpy()).astype(np.float32), M, F)
    c = O.linear(O.a_unlayout(O.from_bfp16(A).astype(np.float32), M, K), O.unpack_b(B, K, 2 * F))
    ref = O.quantize_rows(O.swiglu_from_interleaved(c))[1]
    err, cc = O.max_rel(got, ref), O.corr(got, ref)
    assert err <= 2e-2 and cc > 0.9999, f"max-rel {err:.3e} corr {cc:.6f}"


def test_device_ln_mod(env):
    """npu.run("ln_mod", "glue-ln-m512-s1", [x, branch, params, x', A]) (forward.py:249) with the check_random recipe
    (run_ln.py:89-102): x' bit-exact with run_ln.ln_ref, y within tolerance."""
    torch, npu, ops, dev = env
    M, D, S = 512, 1024, 1
    rng = np.random.default_rng(3)
    x = rng.standard_normal((M, D)).astype(np.float32) * 3
    x[:, rng.integers(0, D, 8)] *= 40
    br = rng.standard_normal((M, D)).astype(np.float32)
    g = np.tanh(rng.standard_normal((2, D))).astype(np.float32)
    sc = (1 + 0.3 * rng.standard_normal((2, D))).astype(np.float32)
    xc = O.bf16_round(O.c_layout_atb(x))                      # run_ln.ln_pack_x
    brc = O.to_bfp16(O.c_layout_atb(br))                      # run_ln.ln_pack_br
    p = O.bf16_round(np.concatenate([g, sc], 1).reshape(-1))  # run_ln.ln_params
    xo = torch.zeros(M * D, dtype=torch.bfloat16, device=dev)
    a = torch.zeros(M * D // 8 * 9, dtype=torch.uint8, device=dev)
    npu.Device().run("ln_mod", f"glue-ln-m{M}-s{S}", [_bf16(torch, xc, dev), _u8(torch, brc, dev),
                                                      _bf16(torch, p, dev), xo, a])
    xp = O.c_unlayout_atb(xo.float().cpu().numpy(), M, D)
    y = O.a_unlayout(O.from_bfp16(a.cpu().numpy()).astype(np.float32), M, D)
    xq = O.c_unlayout_atb(xc, M, D)
    brq = O.c_unlayout_atb(O.from_bfp16(brc).astype(np.float32), M, D)
    gr, scr = np.repeat(g[0:1], M, 0), np.repeat(sc[0:1], M, 0)
    gr[:S * 128], scr[:S * 128] = g[1], sc[1]
    xr, yr = O.ln_ref(xq, brq, gr, scr)
    assert np.array_equal(xp, xr)
    err, c = O.max_rel(y, yr), O.corr(y, yr)
    assert err <= 2e-2 and c > 0.9999, f"y max-rel {err:.3e} corr {c:.6f}"


def test_device_rejects_unmapped_artifacts(env):
    torch, npu, ops, dev = env
    with pytest.raises(NotImplementedError):
        npu.Device().run("attn", "attn32o-v6-s-h32-t8-pf-nk8256-nvrt1", [])
