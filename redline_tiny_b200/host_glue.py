"""Host-side tables and schedule of the DiT, in numpy (computed once per model or per step, as in the reference:
redline/host_glue.py; forward.py:47-61; run_qkv.py:37-50): the sigma schedule and the transformer's timestep, the
Euler update, the sinusoidal frequencies the GPU conditioning kernels read, the joint token layout, the 3-axis RoPE
cos/sin table and the row positions. The per-step conditioning products themselves run on the GPU
(csrc/rl_adaln.cu). Each function cites the reference line it restates; tests pin them against the reference's
outputs.
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


def timestep_freqs(half=128):
    """The sinusoidal embedding's frequencies exp(-ln(10^4) i / half), float32 (host_glue.py:31-36)."""
    return np.exp(-math.log(10000) * np.arange(half, dtype=np.float32) / half)


def joint_layout(vlm_image_mask, n_target=4096, grid=(64, 64)):
    """The joint sequence of the reference's host_glue.joint_layout (host_glue.py:59-65): every text position of the
    VLM sequence is one token, every image slot of it stands for a 2 x 2 patch of latent tokens, and the target
    image's n_target tokens follow. Returns (image_pad_mask, img_shapes): the per-token image flag and one
    (1, h, w) latent grid per image, the target's included. `grid` is that grid (64 x 64 at 1024^2, the only size
    the reference supports; smaller grids serve reduced test configurations)."""
    slots = np.asarray(vlm_image_mask, bool).ravel()
    tokens_per_slot = 1 + 3 * slots.astype(np.int64)              # 1 for text, 4 for an image slot
    is_img = np.concatenate([np.repeat(slots, tokens_per_slot), np.ones(n_target, bool)])
    images = int(is_img.sum()) // n_target
    return is_img, [(1, grid[0], grid[1])] * images


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
