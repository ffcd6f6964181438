"""GPU parity of the VAE decoder convolution (rl_conv2d_bfp16: the packed-weight GEMM on A tiles loaded from the
image by 3-D TMA when W % 128 == 0, else on im2col-gathered rows) against the CPU oracle (oracle/vae_oracle.conv_ref
= vae_ops.conv_ref on the bfp16-rounded activations and weights the reference's vconv multiplies). Output is bf16: max-rel <= 2e-3 + 2^-8 (the GEMM bar plus the output's own bf16 rounding)."""

import numpy as np
import pytest

from oracle import bfp16_oracle as O
from oracle import vae_oracle as VO

pytestmark = pytest.mark.gpu

BF16_OUT_TOL = 2e-3 + 2.0 ** -8


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import ops
    assert torch.cuda.is_available()
    return torch, ops, torch.device("cuda:0")


@pytest.mark.parametrize("H,W,Cin,Cout,k", [(24, 20, 64, 128, 3), (24, 20, 64, 128, 1), (17, 9, 128, 3, 3),
                                            (64, 64, 128, 256, 3), (32, 32, 512, 512, 1),
                                            # the VAE decoder's 288- and 144-channel stages and conv_out (144 -> 4):
                                            # 9 * Cin not a multiple of 64, and a 1x1 conv that needs the gather
                                            (20, 18, 288, 288, 3), (16, 12, 144, 144, 3), (16, 12, 144, 4, 3),
                                            (10, 11, 40, 128, 1),
                                            # W % 128 == 0: the implicit GEMM - 288 channels (5 K steps per tap, the
                                            # last half outside the channel extent), a half-empty last 256-row tile,
                                            # Cout = 256 (the pair kernel), a 1x1 conv over 72 channels; and a 1x1
                                            # conv with Cin % 64 == 0 (its rows are the A rows directly)
                                            (6, 128, 288, 288, 3), (5, 128, 64, 128, 3), (3, 256, 144, 256, 3),
                                            (4, 128, 72, 128, 1), (4, 128, 512, 512, 1)])
def test_conv2d(env, H, W, Cin, Cout, k):
    torch, ops, dev = env
    rng = np.random.default_rng(H * W + Cin + k)
    x = rng.standard_normal((H, W, Cin)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, k, k)) * 0.05).astype(np.float32)
    b = O.bf16_round((rng.standard_normal(Cout) * 0.01).astype(np.float32))
    _, xq = ops.quantize_bfp16(torch.from_numpy(x.reshape(H * W, Cin)).to(dev))
    pw, bias, taps = ops.conv_weight(torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev))
    y = ops.conv2d(xq.view(H, W, Cin), pw, bias, taps)
    ops.device_status()
    got = y.float().cpu().numpy()[:, :, :Cout]
    ref = VO.conv_ref(VO.quantize_pixels(x), VO.decode_conv_b(w), b)
    err = O.max_rel(got, ref)
    assert err <= BF16_OUT_TOL, f"max-rel {err:.3e}"


def test_conv2d_rejects_bad_shapes(env):
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    pw128, _, _ = ops.conv_weight(torch.zeros((128, 128, 3, 3), device=dev))
    with pytest.raises(ValueError):         # weight packed for 128 input channels, input has 64
        ops.conv2d(torch.zeros((4, 4, 64), dtype=torch.bfloat16, device=dev), pw128, None, 3)
    pw, _, _ = ops.conv_weight(torch.zeros((128, 64, 3, 3), device=dev))
    x = torch.zeros((4, 4, 12), dtype=torch.bfloat16, device=dev)
    ws = torch.empty(4 * 4 * 9 * 12 * 2, dtype=torch.uint8, device=dev)
    with pytest.raises(L.RedlineError):     # the C ABI: 12 channels are not whole bfp16 blocks of 8
        L.call("rl_conv2d_bfp16", x.data_ptr(), 4, 4, 12, pw.native.data_ptr(), 128, 3, None, x.data_ptr(),
               ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("H,W,Cin,Cout,k", [(6, 128, 288, 288, 3), (5, 128, 64, 128, 3), (3, 256, 144, 256, 3),
                                            (4, 128, 72, 128, 1)])
def test_conv2d_implicit_equals_gather(env, H, W, Cin, Cout, k):
    """The implicit GEMM (A tiles loaded from the image by 3-D TMA, zero fill as the padding) and the im2col path
    (rl_set_conv_path(1)) multiply the same A rows by the same weights in the same order: bit-identical outputs."""
    torch, ops, dev = env
    from redline_tiny_b200 import _lib as L
    g = torch.Generator(device=dev).manual_seed(H + W + Cin)
    _, xq = ops.quantize_bfp16(torch.randn((H * W, Cin), generator=g, device=dev))
    pw, bias, taps = ops.conv_weight(torch.randn((Cout, Cin, k, k), generator=g, device=dev) * 0.05,
                                     torch.randn(Cout, generator=g, device=dev) * 0.01)
    assert L.lib().rl_conv2d_workspace(H, W, Cin, k) == 0
    y0 = ops.conv2d(xq.view(H, W, Cin), pw, bias, taps)
    prev = L.lib().rl_set_conv_path(1)
    try:
        assert L.lib().rl_conv2d_workspace(H, W, Cin, k) > 0
        y1 = ops.conv2d(xq.view(H, W, Cin), pw, bias, taps)
    finally:
        L.lib().rl_set_conv_path(prev)
    ops.device_status()
    assert torch.equal(y0, y1)
