"""CPU oracle of the VAE decoder convolution - TEST INFRASTRUCTURE ONLY (tests/ import it; the package never does).

Restates redline/vae_ops.py:64-75 (conv_ref: 3x3 pad 1 or 1x1, float64) and the bfp16 rounding the reference's vconv
applies (kernels/vae/vconv.cc:1-17: weights in bfp16 blocks of 8 input channels per output channel and tap, as
vae_ops.pack_vconv packs them, vae_ops.py:44-61; activation strips in bfp16 blocks of 8 channels per pixel), and
decodes pack_vconv's weight stream back to (Cout, Cin, k, k) so the blocking can be compared.
"""

import numpy as np

from . import bfp16_oracle as O


def conv_ref(x, w, b):
    """x (H, W, Cin), w (Cout, Cin, k, k) with k = 3 (pad 1) or 1 -> (H, W, Cout), float64."""
    H, W, _ = x.shape
    k = w.shape[2]
    y = np.zeros((H, W, w.shape[0])) + (0 if b is None else np.asarray(b, np.float64))
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    if k == 1:
        return y + x @ w[:, :, 0, 0].T
    xp = np.zeros((H + 2, W + 2, x.shape[2]))
    xp[1:-1, 1:-1] = x
    for dy in range(3):
        for dx in range(3):
            y += xp[dy:dy + H, dx:dx + W] @ w[:, :, dy, dx].T
    return y


def conv_b(w):
    """The GEMM B operand of a conv weight: B[(dy * k + dx) * Cin + ci][co] = w[co][ci][dy][dx]."""
    cout, cin, k, _ = w.shape
    return np.ascontiguousarray(np.asarray(w, np.float32).transpose(2, 3, 1, 0).reshape(k * k * cin, cout))


def decode_conv_b(w):
    """w rounded as the B200 conv uses it: the bfp16 blocks of pack_b(B), 8 along K (= 8 input channels of one
    tap) in each column of B - the rows of B^T in blocks of 8 (any K % 8 == 0, no tile padding needed)."""
    cout, cin, k, _ = w.shape
    Bd = O.quantize_rows(conv_b(w).T)[1].T
    return Bd.reshape(k, k, cin, cout).transpose(3, 2, 0, 1)


def unpack_vconv_weights(stream, cout, cin, k, kc, nc):
    """Decode pack_vconv's bfp16 weight blocks (vae_ops.py:44-61) back to w (Cout, Cin, k, k); the bias element
    that ends each output-channel chunk is skipped."""
    steps_bytes = k * k * cin * nc // 8 * 9          # per output-channel chunk
    welem = k * kc * nc // 8 * 9
    chunks = np.asarray(stream, np.uint8).reshape(cout // nc, steps_bytes + welem)[:, :steps_bytes]
    vals = O.from_bfp16(chunks.reshape(-1)).reshape(cout // nc, k, cin // kc, nc // 16, k, kc // 8, 2, 8, 8)
    # (co, dy, ci, jp, dx, c8, h, r, c) -> w[co * nc + jp * 16 + h * 8 + r][ci * kc + c8 * 8 + c][dy][dx]
    return vals.transpose(0, 3, 6, 7, 2, 5, 8, 1, 4).reshape(cout, cin, k, k)


def quantize_pixels(x):
    """Activations in bfp16 blocks of 8 channels per pixel (the decoded values)."""
    H, W, C = x.shape
    return O.quantize_rows(np.asarray(x, np.float32).reshape(H * W, C))[1].reshape(H, W, C)
