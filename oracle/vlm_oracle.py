"""CPU oracle of one Qwen3-VL decoder layer - TEST INFRASTRUCTURE ONLY (tests/ import it; the package never does).

Restates the reference's float64 layer check redline/vlm_run.py:458-477 (layer_ref) with its RMS glue rounding
(vlm_run.rms_ref, vlm_run.py:68-71: x' = bf16(x + branch)) and its causal GQA attention (vlm_run.attn_ref,
vlm_run.py:181-190: query head h reads K/V head h // (HQ / HKV), keys above the row masked, first `valid` rows).
Differences from layer_ref, matching the B200 layer's inputs: the weights are the bfp16-decoded B operands the GPU
uses (unpack_b(pack_b(.))), RoPE rotates adjacent pairs (2j, 2j+1) - the reference's packed weights are permuted so
that its NPU kernel does the same - and the residual x2 is rounded to bf16 like the GPU's residual stream.
"""

import numpy as np

from . import bfp16_oracle as O

EPS = 1e-6


def rms(y, w):
    y = np.asarray(y, np.float64)
    return y / np.sqrt((y * y).mean(-1, keepdims=True) + EPS) * w


def rope_pairs(x, cos, sin):
    """Adjacent-pair rotation of (..., rows, 128) by cos / sin (rows, 64)."""
    a, b = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = a * cos - b * sin
    out[..., 1::2] = a * sin + b * cos
    return out


def attention(q, k, v, valid):
    """Causal GQA over the first `valid` rows: q (HQ, n, 128), k / v (HKV, n, 128) -> (n, HQ * 128), rows >= valid
    attend to keys < valid only."""
    hq, n, hd = q.shape
    group = hq // k.shape[0]
    out = np.zeros((n, hq * hd))
    r = np.arange(n)[:, None]
    c = np.arange(n)[None, :]
    mask = (c > np.minimum(r, valid - 1)) | (c >= valid)
    for h in range(hq):
        s = q[h] @ k[h // group].T / np.sqrt(hd)
        s[mask] = -np.inf
        w = np.exp(s - s.max(1, keepdims=True))
        out[:, h * hd:(h + 1) * hd] = (w / w.sum(1, keepdims=True)) @ v[h // group]
    return out


def decode_b(B):
    """The weights the GPU multiplies with: B rounded to bfp16 in pack_b's blocks (8 along K)."""
    K, N = B.shape
    return O.unpack_b(O.pack_b(np.asarray(B, np.float32)), K, N).astype(np.float64)


def layer(x, lw, cos, sin, valid, heads, kv_heads, branch=None):
    """One decoder layer on float inputs; lw holds numpy float32 arrays shaped as vlm.random_lm_weights makes
    them. Returns x_out = x2 + down (float64) over all rows."""
    M, D = x.shape
    hd = 128
    br = np.zeros_like(x) if branch is None else branch
    x1 = O.bf16_round((np.asarray(x, np.float32) + np.asarray(br, np.float32)).astype(np.float32)).astype(np.float64)
    h = rms(x1, lw["w_in"])
    qkv = h @ decode_b(lw["qkv"])
    q = qkv[:, :heads * hd].reshape(M, heads, hd).transpose(1, 0, 2)
    k = qkv[:, heads * hd:(heads + kv_heads) * hd].reshape(M, kv_heads, hd).transpose(1, 0, 2)
    v = qkv[:, (heads + kv_heads) * hd:].reshape(M, kv_heads, hd).transpose(1, 0, 2)
    q = rope_pairs(rms(q, lw["q_norm"]), cos, sin)
    k = rope_pairs(rms(k, lw["k_norm"]), cos, sin)
    o = attention(q, k, v, valid)
    x2 = O.bf16_round((x1 + o @ decode_b(lw["o"])).astype(np.float32)).astype(np.float64)
    h2 = rms(x2, lw["w_post"])
    gt = h2 @ decode_b(lw["gate"].T)
    up = h2 @ decode_b(lw["up"].T)
    return x2 + (gt / (1 + np.exp(-gt)) * up) @ decode_b(lw["down"])
