"""CPU restatement of the DiT's per-step adaLN conditioning - TEST INFRASTRUCTURE ONLY (imported by tests/ and the
DiT oracle, never by the product package, which runs this conditioning on the GPU: csrc/rl_adaln.cu).

The reference computes these small products on the host in numpy float32 (redline/host_glue.py:31-48; the
LayerNorm parameter rows forward.py:231-238). Each function cites the line it restates; tests/test_oracle_golden.py
pins them bit for bit against the reference's own outputs (tests/golden), and tests/test_gpu_adaln.py holds the
GPU kernels to them.
"""

import numpy as np

from redline_tiny_b200.host_glue import timestep_freqs


def silu(x):
    return x / (1 + np.exp(-x))


def _affine(x, w, b=None):
    """x @ w^T (+ b), float32: the reference's torch-layout linear on the host."""
    y = x @ w.T
    return y + b if b is not None else y


def temb(w, t):
    """Timestep embedding on rows [t, 0] (host_glue.py:31-40): the sinusoidal features of t * 1000 (cos half, then
    sin half), linear_1, SiLU, linear_2."""
    rows = np.array([t, 0.0], np.float32) * 1000.0
    arg = rows[:, None] * timestep_freqs()[None]
    feats = np.concatenate([np.cos(arg), np.sin(arg)], -1).astype(np.float32)
    pre = "time_text_embed.timestep_embedder."
    hidden = silu(_affine(feats, w[pre + "linear_1.weight"], w.get(pre + "linear_1.bias")))
    return _affine(hidden, w[pre + "linear_2.weight"], w.get(pre + "linear_2.bias"))


def modulation(w, te):
    """(2, 4 * HID) = [scale1 | gate1 | scale2 | gate2] = modulation.1(SiLU(temb)) (host_glue.py:43-44)."""
    return _affine(silu(te), w["modulation.1.weight"])


def norm_out_scale(w, te):
    """norm_out.linear(SiLU(temb)) (host_glue.py:47-48)."""
    return _affine(silu(te), w["norm_out.linear.weight"])


def adaln_params(mod, out_scale, D):
    """The LayerNorm parameter sets of one step (forward.py:231-238), float32 (2, 2, D) = rows [g | sc] before their
    bf16 rounding: first (1, 1 + scale1), mlp (tanh gate1, 1 + scale2), attn (tanh gate2, 1 + scale1),
    out (tanh gate2, 1 + out_scale); mod = [scale1 | gate1 | scale2 | gate2]."""
    s1, g1, s2, g2 = (np.asarray(mod[:, i * D:(i + 1) * D], np.float32) for i in range(4))
    out_scale = np.asarray(out_scale[:, :D], np.float32)

    def rows(g, sc):
        return np.concatenate([np.asarray(g, np.float32), np.asarray(sc, np.float32)], 1).reshape(2, 2, D)
    return {"first": rows(np.ones((2, D)), 1 + s1), "mlp": rows(np.tanh(g1), 1 + s2),
            "attn": rows(np.tanh(g2), 1 + s1), "out": rows(np.tanh(g2), 1 + out_scale)}
