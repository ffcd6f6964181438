"""CPU oracle of the DiT denoise step (config 4) - TEST INFRASTRUCTURE ONLY (imported by tests/ and bench.py's CPU
legs, never by the product package).

Composes the restated reference ops of bfp16_oracle.py in the order of the reference's block loop
(redline/forward.py:240-254) and step (forward.py:396-412, 256-269, 58-61), rounding where the stored tensors are
rounded: GEMM outputs and QK-norm/RoPE outputs to bf16, LayerNorm outputs, the attention output and the SwiGLU output
to bfp16 (blocks of 8 along the row), exactly as the GPU pipeline stores them. The adaLN modulation comes from
oracle/host_oracle.py, the RoPE table and token layout from the host glue the product uses
(redline_tiny_b200.host_glue); both are pinned against the reference by tests/golden.
"""

import math

import numpy as np

from . import bfp16_oracle as O
from . import host_oracle as HO

HEAD_DIM = 128
C_LOG2 = math.log2(math.e) / math.sqrt(HEAD_DIM)


def decode_b(B):
    """Float B (K, N) -> its bfp16-decoded values (blocks of 8 consecutive K per column), as pack_b + from_bfp16
    produce them, without the layout permutation."""
    B = np.ascontiguousarray(np.asarray(B, np.float32).T)
    return O.quantize_rows(B)[1].T.copy()


def interleave_up(gate, proj):
    return O.interleave_up(gate, proj)


def prepare(weights):
    """Torch/numpy float weights (dit.random_weights layout) -> decoded numpy operands."""
    def n(t):
        return t.detach().cpu().numpy() if hasattr(t, "numpy") else np.asarray(t)
    blocks = []
    for b in weights["blocks"]:
        blocks.append({
            "qkv": decode_b(n(b["qkv"])), "o": decode_b(n(b["o"])),
            "up": decode_b(interleave_up(n(b["gate"]), n(b["proj"]))),
            "down": decode_b(n(b["down"])),
            "wq": (n(b["norm_q"]).astype(np.float32) * np.float32(C_LOG2)).astype(np.float32),
            "wk": n(b["norm_k"]).astype(np.float32),
        })
    return {"blocks": blocks, "img_in": decode_b(n(weights["img_in"])), "proj_out": decode_b(n(weights["proj_out"])),
            "host": weights["host"]}


def _ln(x, br, p, split):
    """ln_ref with per-row parameters (rows < split use row 1); returns (x' bf16, y rounded to bfp16)."""
    M = x.shape[0]
    g = np.repeat(p[0:1, 0], M, 0)
    sc = np.repeat(p[0:1, 1], M, 0)
    g[:split], sc[:split] = p[1, 0], p[1, 1]
    xp, y = O.ln_ref(x, br, g, sc)
    return xp, O.quantize_rows(y.astype(np.float32))[1]


def forward(cfg, prep, latents, text_states, sigma, host_glue, reduce=None):
    """The step's velocity. With tensor-parallel shards in `prep`, `reduce` sums a partial (M, D) float32
    projection output over the ranks (an all-reduce) before it is rounded to bf16."""
    D, M, T = cfg.hidden, cfg.M, cfg.text
    reduce = reduce or (lambda c: c)
    te = HO.temb(prep["host"], host_glue.model_t(sigma))
    mod = HO.modulation(prep["host"], te)
    out_scale = HO.norm_out_scale(prep["host"], te)
    s1, g1, s2, g2 = (mod[:, i * D:(i + 1) * D] for i in range(4))

    def lp(g, sc):
        return O.bf16_round(np.stack([np.asarray(g, np.float32), np.asarray(sc, np.float32)], 1))  # (2, 2, D)
    p_first, p_mlp = lp(np.ones((2, D)), 1 + s1), lp(np.tanh(g1), 1 + s2)
    p_attn, p_out = lp(np.tanh(g2), 1 + s1), lp(np.tanh(g2), 1 + out_scale)
    pad, shapes = host_glue.joint_layout(np.zeros(T, bool), n_target=cfg.image, grid=cfg.grid)
    rot = host_glue.rope(pad, shapes)
    cos, sin = rot[..., 0], rot[..., 1]

    lat = O.quantize_rows(O.bf16_round(np.asarray(latents, np.float32)))[1]
    emb = np.empty((M, D), np.float32)
    emb[:T] = O.bf16_round(np.asarray(text_states, np.float32))
    emb[T:] = O.bf16_round(O.linear(lat, prep["img_in"]))
    x0, a = _ln(emb, np.zeros_like(emb), p_first, T)
    for i, b in enumerate(prep["blocks"]):
        H = b["qkv"].shape[1] // (3 * HEAD_DIM)       # heads on this rank
        qkv = O.bf16_round(O.linear(a, b["qkv"]))
        o = np.empty((M, H * HEAD_DIM), np.float32)
        for h in range(H):
            q = O.bf16_round(O.rms_rope(qkv[:, h * 128:(h + 1) * 128], b["wq"], cos, sin))
            k = O.bf16_round(O.rms_rope(qkv[:, (H + h) * 128:(H + h + 1) * 128], b["wk"], cos, sin))
            v = qkv[:, (2 * H + h) * 128:(2 * H + h + 1) * 128]
            # q already carries log2(e)/sqrt(128): logits in log2 units, softmax base 2 == base e of q.k/sqrt(d)
            o[:, h * 128:(h + 1) * 128] = O.attention_f64(q * np.float32(math.sqrt(HEAD_DIM) / math.log2(math.e)),
                                                          k, v)
        o = O.quantize_rows(o)[1]
        c = O.bf16_round(reduce(O.linear(o, b["o"])))
        x1, a = _ln(x0, c, p_mlp, T)
        hsw = O.quantize_rows(O.swiglu_from_interleaved(O.linear(a, b["up"])))[1]
        c = O.bf16_round(reduce(O.linear(hsw, b["down"])))
        x0, a = _ln(x1, c, p_out if i == len(prep["blocks"]) - 1 else p_attn, T)
    v = O.linear(a[T:], prep["proj_out"])
    return v[:, :cfg.latent_ch]
