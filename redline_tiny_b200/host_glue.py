"""Per-step host glue of the DiT, on the CPU in numpy float32 (tiny matvecs and tables).

These run on the host in the reference as well (redline/host_glue.py; forward.py:47-61; run_qkv.py:37-50). They
produce the inputs of the GPU epilogues: the adaLN gate / scale rows, the 3-axis RoPE cos/sin table and the row
positions. Each function cites the reference line it restates; tests pin them against the reference's outputs.
"""

import math

import numpy as np

# The model's distilled sigma schedule (forward.py:48).
SIGMAS = [1.0, 0.978453, 0.95418, 0.926626, 0.89508, 0.845148, 0.704534, 0.414568]


def _bf16(x):
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def model_t(sigma):
    """The timestep the transformer sees: bf16(bf16(sigma * 1000) / 1000) (forward.py:51-55)."""
    t = _bf16(np.float32(sigma * 1000))
    return float(_bf16(np.float32(t) / np.float32(1000)))


def euler(latents, v, i, sigmas=SIGMAS):
    """Flow-matching Euler step i (forward.py:58-61)."""
    nxt = sigmas[i + 1] if i + 1 < len(sigmas) else 0.0
    return latents + (nxt - sigmas[i]) * v


def silu(x):
    return x / (1 + np.exp(-x))


def _linear(x, w, b=None):
    y = x @ w.T
    return y + b if b is not None else y


def timestep_freqs(half=128):
    """The sinusoidal embedding's frequencies exp(-ln(10^4) i / half), float32 (host_glue.py:31-36)."""
    return np.exp(-math.log(10000) * np.arange(half, dtype=np.float32) / half)


def temb(w, t):
    """Sinusoidal(256) -> linear_1 -> SiLU -> linear_2 on rows [t, 0] (host_glue.py:31-40)."""
    ts = np.array([t, 0.0], np.float32) * 1000.0
    freqs = timestep_freqs()
    arg = ts[:, None] * freqs[None]
    e = np.concatenate([np.cos(arg), np.sin(arg)], -1).astype(np.float32)
    p = "time_text_embed.timestep_embedder."
    h = silu(_linear(e, w[p + "linear_1.weight"], w.get(p + "linear_1.bias")))
    return _linear(h, w[p + "linear_2.weight"], w.get(p + "linear_2.bias"))


def modulation(w, te):
    """Linear(SiLU(temb)) -> (2, 4 * HID) = [scale1 | gate1 | scale2 | gate2] (host_glue.py:43-44)."""
    return _linear(silu(te), w["modulation.1.weight"])


def norm_out_scale(w, te):
    """host_glue.py:47-48."""
    return _linear(silu(te), w["norm_out.linear.weight"])


def adaln_params(mod, out_scale, D):
    """The LayerNorm parameter sets of one step (forward.py:231-238), float32 (2, 2, D) = rows [g | sc] before their
    bf16 rounding: first (1, 1 + scale1), mlp (tanh gate1, 1 + scale2), attn (tanh gate2, 1 + scale1),
    out (tanh gate2, 1 + out_scale); mod = [scale1 | gate1 | scale2 | gate2]."""
    s1, g1, s2, g2 = (np.asarray(mod[:, i * D:(i + 1) * D], np.float32) for i in range(4))
    out_scale = np.asarray(out_scale[:, :D], np.float32)

    def lp(g, sc):
        return np.concatenate([np.asarray(g, np.float32), np.asarray(sc, np.float32)], 1).reshape(2, 2, D)
    return {"first": lp(np.ones((2, D)), 1 + s1), "mlp": lp(np.tanh(g1), 1 + s2),
            "attn": lp(np.tanh(g2), 1 + s1), "out": lp(np.tanh(g2), 1 + out_scale)}


def joint_layout(vlm_image_mask, n_target=4096, grid=(64, 64)):
    """The joint sequence: text positions, image slots expanded to 2x2 latent tokens, then the target's tokens
    (host_glue.py:59-65). Returns (image_pad_mask, img_shapes). `grid` is the latent token grid of each image
    (64 x 64 at 1024^2, the only size the reference supports; smaller grids serve reduced test configurations)."""
    m = np.concatenate([np.asarray(vlm_image_mask, bool).ravel(), np.ones(n_target // 4, bool)])
    pad = np.repeat(m, np.where(m, 4, 1))
    return pad, [(1, grid[0], grid[1])] * (int(pad.sum()) // n_target)


def rope(image_pad_mask, img_shapes, axes=(16, 56, 56), theta=10000):
    """3-axis RoPE table (seq, 64, 2) = (cos, sin) (host_glue.py:68-91): text tokens advance one shared position
    on all three axes; each image block freezes the frame axis and lays out a centred h x w grid."""
    is_img = np.asarray(image_pad_mask, bool)
    n = is_img.size
    frame = np.empty(n, np.int64)
    hidx = np.empty(n, np.int64)
    widx = np.empty(n, np.int64)
    cursor = pos = 0
    for _, h, w in img_shapes:
        start = cursor + int(np.argmax(is_img[cursor:]))
        run = start - cursor
        frame[cursor:start] = pos + np.arange(run)
        pos += run
        frame[start:start + h * w] = pos
        pos += max(h, w)
        ys = np.arange(-(h - h // 2), h // 2)
        xs = np.arange(-(w - w // 2), w // 2)
        hidx[start:start + h * w] = np.repeat(ys, w)
        widx[start:start + h * w] = np.tile(xs, h)
        cursor = start + h * w
    if cursor < n:
        frame[cursor:] = pos + np.arange(n - cursor)
    text = ~is_img
    hidx[text] = frame[text]
    widx[text] = frame[text]
    ang = [np.outer(idx, 1.0 / theta ** (np.arange(0, d, 2, dtype=np.float32) / d))
           for idx, d in zip((frame, hidx, widx), axes)]
    a = np.concatenate(ang, -1)
    return np.stack([np.cos(a), np.sin(a)], -1).astype(np.float32)


def positions(M, P=4128):
    """RoPE row per GEMM row, -1 = pad (run_qkv.py:37-50): M 4096 = the cached step's target rows; M 8704 / 4608 =
    step 1's [prefix P | pad | target 4096 from row 4224 / 512 | pad]."""
    if M == 4096:
        return P + np.arange(4096)
    if M in (8704, 4608):
        row0 = 4224 if M == 8704 else 512
        pos = np.full(M, -1)
        pos[:P] = np.arange(P)
        pos[row0:row0 + 4096] = P + np.arange(4096)
        return pos
    raise ValueError(M)
