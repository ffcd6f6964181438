"""Run one hot-path kernel (or one DiT block) on its benchmark-config shape a few times - the target of ncu captures.

    python -m redline_tiny_b200.profile_cases <case> [--iters N]

cases: linear_c1 | quantize_c1 | swiglu_up_c2 | attention_c3 | qkv_post_c3 | ln_mod_c4 | dit_block_c4 |
       vae_conv_128x1152 | vae_conv_512x288 (3x3 convs of the VAE decoder: the implicit GEMM)
Inputs are seeded synthetic tensors of the configs' shapes (a few hundred MB on the device at most).
"""

import argparse
import time

import torch

from . import _lib as L
from . import dit, ops


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    s = torch.cuda.current_stream().cuda_stream
    c = args.case
    if c in ("linear_c1", "quantize_c1"):
        M, K, N = 4352, 3072, 12288
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        dq = torch.empty_like(x)
        w = ops.PackedWeight.from_float(torch.randn((K, N), generator=g, device=dev) * 0.02)
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

        def fn():
            L.call("rl_quantize_bfp16", x.data_ptr(), L.RL_BF16, M, K, L.RL_ROWMAJOR, None, dq.data_ptr(), s)
            if c == "linear_c1":
                L.call("rl_linear_bfp16", dq.data_ptr(), M, K, w.native.data_ptr(), N, None, L.RL_EPI_NONE,
                       out.data_ptr(), L.RL_BF16, s)
    elif c == "swiglu_up_c2":
        M, K, F = 512, 4096, 12288
        x = ops.quantize_bfp16(torch.randn((M, K), generator=g, device=dev), want_bytes=False)[1]
        w = ops.PackedWeight.from_float(torch.randn((K, 2 * F), generator=g, device=dev) * 0.02, swiglu=True)
        h = torch.empty((M, F), dtype=torch.bfloat16, device=dev)

        def fn():
            ops.swiglu_up(x, w, out=h)
    elif c in ("vae_conv_128x1152", "vae_conv_512x288"):
        H, C = (128, 1152) if c == "vae_conv_128x1152" else (512, 288)
        x = ops.quantize_bfp16(torch.randn((H * H, C), generator=g, device=dev), want_bytes=False)[1].view(H, H, C)
        pw, bias, taps = ops.conv_weight(torch.randn((C, C, 3, 3), generator=g, device=dev) * 0.02,
                                         torch.randn(C, generator=g, device=dev) * 0.01)
        y = torch.empty((H, H, pw.N), dtype=torch.bfloat16, device=dev)

        def fn():
            ops.conv2d(x, pw, bias, taps, out=y)
    elif c in ("attention_c3", "qkv_post_c3", "ln_mod_c4", "dit_block_c4"):
        cfg = dit.DiTConfig(blocks=1)
        model = dit.DiT(cfg, dit.random_weights(cfg, seed=0))
        model.set_t(0.5)
        model.embed(torch.randn((cfg.image, cfg.latent_ch), generator=g, device=dev),
                    torch.randn((cfg.text, cfg.hidden), generator=g, device=dev))
        b = model.blocks[0]
        model._linear(model.a, b["qkv"], model.qkv)

        def qkv_post():
            L.call("rl_qkv_post", model.qkv.data_ptr(), model.rope_cs.data_ptr(), b["wq"].data_ptr(),
                   b["wk"].data_ptr(), cfg.M, cfg.heads, model.q.data_ptr(), model.k.data_ptr(), model.vt.data_ptr(),
                   model.ldv, s)
        qkv_post()

        def attention():
            L.call("rl_attention", model.q.data_ptr(), model.k.data_ptr(), model.vt.data_ptr(), model.ldv, cfg.heads,
                   cfg.M, cfg.M, cfg.M, None, 1.0, model.o.data_ptr(), cfg.hidden, s)
        attention()
        model._linear(model.o, b["o"], model.c)
        fn = {"attention_c3": attention, "qkv_post_c3": qkv_post,
              "ln_mod_c4": lambda: model._ln(model.x[0], model.c, model.params["mlp"], model.x[1], model.a),
              "dit_block_c4": lambda: model.block(0)}[c]
    else:
        raise SystemExit(f"unknown case {c}")
    for _ in range(args.iters):
        fn()
    torch.cuda.synchronize()
    t = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    print(f"{c}: last call {1e3 * (time.perf_counter() - t):.3f} ms wall", flush=True)
    L.device_status()


if __name__ == "__main__":
    main()
