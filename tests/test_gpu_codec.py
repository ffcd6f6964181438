"""GPU parity of the bfp16 codec kernels against the CPU oracle: bit-exact bytes and values."""

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


def test_quantize_golden_fp32_edge_cases(env, golden):
    torch, ops, dev = env
    x = golden["quant_in"].reshape(-1, 8)
    q, dq = ops.quantize_bfp16(torch.from_numpy(x).to(dev))
    assert np.array_equal(q.cpu().numpy(), golden["quant_out"])
    ref = O.from_bfp16(golden["quant_out"]).astype(np.float32).reshape(x.shape)
    got = dq.float().cpu().numpy()
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin], ref[fin])
    ops.device_status()


def test_quantize_golden_bf16_inputs(env, golden):
    torch, ops, dev = env
    x = golden["quant_bf16_in"].reshape(-1, 64)
    q, _ = ops.quantize_bfp16(_bf16(torch, x, dev))
    assert np.array_equal(q.cpu().numpy(), golden["quant_bf16_out"])


@pytest.mark.parametrize("M,K", [(1, 8), (3, 24), (33, 64), (128, 64), (4352, 3072)])
def test_quantize_rowmajor_random(env, M, K):
    torch, ops, dev = env
    rng = np.random.default_rng(M * 7 + K)
    x = (rng.standard_normal((M, K)) * np.exp2(rng.integers(-30, 30, (M, 1)))).astype(np.float32)
    for xt, xr in ((torch.from_numpy(x).to(dev), x), (_bf16(torch, x, dev), O.bf16_round(x))):
        q, dq = ops.quantize_bfp16(xt)
        ref = O.to_bfp16(xr)
        assert np.array_equal(q.cpu().numpy(), ref)
        assert np.array_equal(dq.float().cpu().numpy(), O.from_bfp16(ref).astype(np.float32).reshape(M, K))
    ops.device_status()


@pytest.mark.parametrize("M,K", [(128, 64), (256, 192), (4352, 3072)])
def test_quantize_a_layout(env, M, K):
    torch, ops, dev = env
    rng = np.random.default_rng(11)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    q, dq = ops.quantize_bfp16(_bf16(torch, x, dev), layout="a_layout")
    assert np.array_equal(q.cpu().numpy(), O.to_bfp16(O.a_layout(x)))
    assert np.array_equal(dq.float().cpu().numpy(), O.quantize_rows(x)[1])


@pytest.mark.parametrize("layout", ["rowmajor", "a_layout"])
def test_dequantize(env, golden, layout):
    torch, ops, dev = env
    M, K = 256, 128
    rng = np.random.default_rng(3)
    raw = rng.integers(0, 256, (M * K // 8, 9)).astype(np.uint8)
    raw[:, 0] = rng.integers(0, 238, M * K // 8)
    raw = raw.reshape(-1)
    vals = O.from_bfp16(raw).astype(np.float32)
    ref = vals.reshape(M, K) if layout == "rowmajor" else O.a_unlayout(vals, M, K)
    rt = torch.from_numpy(raw).to(dev)
    for dt in (torch.float32, torch.bfloat16):
        got = ops.dequantize_bfp16(rt, M, K, layout=layout, dtype=dt).float().cpu().numpy()
        assert np.array_equal(got, ref)
    # golden decoder vectors (exponents 0..254)
    d = golden["dec_in"]
    got = ops.dequantize_bfp16(torch.from_numpy(d).to(dev), 1, d.size // 9 * 8).cpu().numpy().ravel()
    ref = golden["dec_out"].astype(np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin], ref[fin])


@pytest.mark.parametrize("K,N", [(128, 256), (3072, 1024)])
def test_pack_b_bit_exact(env, golden, K, N):
    torch, ops, dev = env
    if K == 128:
        W = golden["pack_in"]
        ref = golden["pack_out"]
    else:
        W = (np.random.default_rng(0).standard_normal((K, N)) * 0.02).astype(np.float32)
        ref = O.pack_b(W)
    got = ops.pack_b(torch.from_numpy(W).to(dev)).cpu().numpy()
    assert np.array_equal(got, ref)
    gotb = ops.pack_b(_bf16(torch, W, dev)).cpu().numpy()
    assert np.array_equal(gotb, O.pack_b(O.bf16_round(W)))


@pytest.mark.parametrize("swiglu", [False, True])
def test_native_repack_consistent(env, swiglu):
    torch, ops, dev = env
    K, N = 256, 512
    W = (np.random.default_rng(1).standard_normal((K, N)) * 0.02).astype(np.float32)
    a = ops.PackedWeight.from_pack_b(torch.from_numpy(O.pack_b(W)).to(dev), K, N, swiglu=swiglu).native
    b = ops.PackedWeight.from_float(torch.from_numpy(W).to(dev), swiglu=swiglu).native
    assert torch.equal(a, b)
    # same bytes, regrouped: the multiset of (exponent, mantissa) blocks is preserved per tile
    assert a.numel() == K * N // 8 * 9
    ops.device_status()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("M,K", [(4352, 3072), (77, 40), (1, 8)])
def test_decoded_only_quantiser_equals_full_quantiser(M, K, dtype):
    """The decoded-only row-major quantiser (the GEMM's A operand; an unrolled kernel of its own) writes exactly the
    decoded values of the full quantiser (bytes + decoded), whose bytes are bit-exact against the oracle above;
    ragged block counts included."""
    import torch
    from redline_tiny_b200 import ops
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(M + K)
    x = torch.from_numpy((rng.standard_normal((M, K)) * np.exp2(rng.integers(-20, 20, (M, 1)))).astype(np.float32))
    x = x.to(dev) if dtype == "f32" else x.to(dev).to(torch.bfloat16)
    q, dq_full = ops.quantize_bfp16(x)
    _, dq_only = ops.quantize_bfp16(x, want_bytes=False)
    ops.device_status()
    assert torch.equal(dq_only, dq_full)
    ref = O.from_bfp16(O.to_bfp16(x.float().cpu().numpy().reshape(-1))).astype(np.float32).reshape(M, K)
    assert np.array_equal(dq_only.float().cpu().numpy(), ref)
