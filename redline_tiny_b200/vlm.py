"""Qwen3-VL text-encoder decoder layer on B200, composed from the hot-path kernels.

Follows the reference's LM._layer (redline/vlm_run.py:396-431) and its float64 check layer_ref (vlm_run.py:458-477):

    x1, a1 = rms_mod(x0, branch, w_in)          x1 = bf16(x0 + branch); a1 = RMSNorm(x1) * w_in, bfp16
    qkv = a1 @ Wqkv                              N = (HQ + 2 HKV) * 128
    q, k, vt = qkv_post_gqa(qkv)                 q / k RMSNorm * w (q also * log2e / sqrt(128)), adjacent-pair RoPE
    o = attention_gqa(q, k, vt)                  causal, query head h reads K/V head h / (HQ / HKV)
    c = o @ Wo
    x2, a2 = rms_mod(x1, c, w_post)
    h = SwiGLU(a2 @ Wup)                          fused into the up GEMM ([gate 64 | proj 64] per 128 columns)
    branch = h @ Wdown                            x_out = x2 + branch, folded into the next layer's rms_mod

The q / k norm weights are taken in the RoPE-pair order the reference packs them in (adjacent pairs 2j, 2j+1,
vlm_run.balance_qk), so RoPE rotates adjacent pairs. Rows at or after `valid` (the prompt length) are padding: they
attend to the valid keys only and their outputs are not used.
"""

import math

import torch

from . import ops
from . import _lib as L
from .dit import interleave_up_torch

HEAD_DIM = 128
C_LOG2 = math.log2(math.e) / math.sqrt(HEAD_DIM)


class LMConfig:
    """Qwen3-VL-8B text decoder defaults (vlm_run.py:22-23): hidden 4096, 32 query heads, 8 K/V heads, FFN 12288."""

    def __init__(self, hidden=4096, heads=32, kv_heads=8, ffn=12288, layers=1):
        assert hidden % 128 == 0 and heads % kv_heads == 0
        self.hidden, self.heads, self.kv_heads, self.ffn, self.layers = hidden, heads, kv_heads, ffn, layers

    def flop_per_layer(self, M, valid):
        D, F, H, Hk = self.hidden, self.ffn, self.heads, self.kv_heads
        return (2 * M * D * (H + 2 * Hk) * 128 + 2 * M * H * 128 * D + 2 * M * D * 2 * F + 2 * M * F * D
                + 2 * H * valid * (valid + 1) * 128)


def random_lm_weights(cfg, seed=0, device="cuda"):
    """Random-init layer weights (no checkpoint): linears N(0, 0.02) as B = W^T (K, N); RMS weights N(1, 0.1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    D, F, H, Hk = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads

    def randn(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device=device) * std).float()

    layers = []
    for _ in range(cfg.layers):
        layers.append({
            "qkv": randn(D, (H + 2 * Hk) * HEAD_DIM), "o": randn(H * HEAD_DIM, D),
            "gate": randn(F, D), "up": randn(F, D), "down": randn(F, D),
            "w_in": 1 + randn(D, std=0.1), "w_post": 1 + randn(D, std=0.1),
            "q_norm": 1 + randn(HEAD_DIM, std=0.1), "k_norm": 1 + randn(HEAD_DIM, std=0.1),
        })
    return {"layers": layers}


def rms_params(w):
    """rms_mod parameter rows [g | sc] x 2 with g = 1 (vlm_run.rms_params), bf16 (2 * 2D)."""
    row = torch.cat([torch.ones_like(w), w]).float()
    return torch.cat([row, row]).to(torch.bfloat16).contiguous()


class LM:
    """Resident packed weights and preallocated buffers for `cfg.layers` decoder layers over M rows."""

    def __init__(self, cfg, weights, M, device="cuda", fuse_qkv=True):
        self.cfg, self.M = cfg, M
        dev = torch.device(device)
        self.dev = dev
        D, F, H, Hk = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads
        pw = ops.PackedWeight.from_float
        self.layers = []
        for lw in weights["layers"]:
            self.layers.append({
                "qkv": pw(lw["qkv"].to(dev)), "o": pw(lw["o"].to(dev)),
                "up": pw(interleave_up_torch(lw["gate"], lw["up"]).to(dev), swiglu=True),
                "down": pw(lw["down"].to(dev)),
                "p_in": rms_params(lw["w_in"].to(dev)), "p_post": rms_params(lw["w_post"].to(dev)),
                "wq": (lw["q_norm"] * C_LOG2).to(dev).float().contiguous(),
                "wk": lw["k_norm"].to(dev).float().contiguous(),
            })
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = [torch.empty(M, D, **bf) for _ in range(3)]
        self.a = torch.empty(M, D, **bf)
        self.qkv = torch.empty(M, (H + 2 * Hk) * HEAD_DIM, **bf)
        self.ldv = (M + 127) // 128 * 128
        self.fuse_qkv = fuse_qkv   # QK-RMSNorm + RoPE in the QKV GEMM's epilogue (rl_qkv_linear)
        self.q = torch.empty(H, M, HEAD_DIM, **bf)
        self.k = torch.empty(Hk, M, HEAD_DIM, **bf)
        self.vt = torch.zeros(Hk, HEAD_DIM, self.ldv, **bf)
        self.o = torch.empty(M, H * HEAD_DIM, **bf)
        self.c = [torch.empty(M, D, **bf) for _ in range(2)]
        self.h = torch.empty(M, F, **bf)
        self.row_limit = None
        self.valid = M

    def set_positions(self, cos, sin, valid):
        """RoPE table (cos, sin per adjacent pair; cos / sin: (M, 64)) and the prompt length: causal row limits."""
        M = self.M
        cs = torch.stack([torch.as_tensor(cos, dtype=torch.float32), torch.as_tensor(sin, dtype=torch.float32)], -1)
        self.rope_cs = cs.reshape(M, 128).to(self.dev).contiguous()
        r = torch.arange(M, dtype=torch.int32)
        self.row_limit = torch.minimum(r, torch.tensor(valid - 1, dtype=torch.int32)).to(self.dev)
        self.valid = int(valid)

    def load_x(self, x):
        self.x[0].copy_(torch.as_tensor(x).to(self.dev, torch.bfloat16))
        self.cur, self.br = 0, None

    def _linear(self, x, w, out, epi=L.RL_EPI_NONE):
        L.call("rl_linear_bfp16", x.data_ptr(), x.shape[0], x.shape[1], w.native.data_ptr(), w.N, None, epi,
               out.data_ptr(), L.RL_BF16, torch.cuda.current_stream().cuda_stream)

    def _rms(self, x, br, p, xo, a):
        s = torch.cuda.current_stream().cuda_stream
        L.call("rl_rms_mod", x.data_ptr(), None if br is None else br.data_ptr(), L.RL_BF16, p.data_ptr(), self.M,
               self.cfg.hidden, 0, xo.data_ptr(), a.data_ptr(), None, s)

    def layer(self, i):
        cfg, lw, M = self.cfg, self.layers[i], self.M
        s = torch.cuda.current_stream().cuda_stream
        x0, x1, x2 = self.x[self.cur], self.x[(self.cur + 1) % 3], self.x[(self.cur + 2) % 3]
        self._rms(x0, self.br, lw["p_in"], x1, self.a)
        if self.fuse_qkv:   # QK-RMSNorm + RoPE in the QKV GEMM's epilogue
            L.call("rl_qkv_linear", self.a.data_ptr(), M, cfg.hidden, lw["qkv"].native.data_ptr(), cfg.heads,
                   cfg.kv_heads, self.rope_cs.data_ptr(), lw["wq"].data_ptr(), lw["wk"].data_ptr(),
                   self.q.data_ptr(), self.k.data_ptr(), self.vt.data_ptr(), self.ldv, s)
        else:
            self._linear(self.a, lw["qkv"], self.qkv)
            L.call("rl_qkv_post_gqa", self.qkv.data_ptr(), self.rope_cs.data_ptr(), lw["wq"].data_ptr(),
                   lw["wk"].data_ptr(), M, cfg.heads, cfg.kv_heads, self.q.data_ptr(), self.k.data_ptr(),
                   self.vt.data_ptr(), self.ldv, s)
        L.call("rl_attention_gqa", self.q.data_ptr(), self.k.data_ptr(), self.vt.data_ptr(), self.ldv, cfg.heads,
               cfg.kv_heads, M, M, self.valid, self.row_limit.data_ptr(), 1.0, self.o.data_ptr(),
               cfg.heads * HEAD_DIM, s)
        c = self.c[0]
        self._linear(self.o, lw["o"], c)
        self._rms(x1, c, lw["p_post"], x2, self.a)
        self._linear(self.a, lw["up"], self.h, epi=L.RL_EPI_SWIGLU)
        cd = self.c[1]
        self._linear(self.h, lw["down"], cd)
        self.cur, self.br = (self.cur + 2) % 3, cd

    def x_out(self):
        """The residual stream after the last layer run (x2 + down) through one more glue pass."""
        x0, x1 = self.x[self.cur], self.x[(self.cur + 1) % 3]
        self._rms(x0, self.br, self.layers[-1]["p_in"], x1, self.a)
        return x1
