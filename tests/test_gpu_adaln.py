"""GPU adaLN conditioning (rl_sinusoidal_embed, rl_matvec_f32, rl_adaln_params) against the host glue and the
reference's golden vectors for t = 0.5 (host_glue.py:31-48, forward.py:231-238: timestep embedding, modulation,
norm_out, LayerNorm parameter rows)."""

import numpy as np
import pytest

from oracle import host_oracle as HO
from redline_tiny_b200 import host_glue as HG

pytestmark = pytest.mark.gpu

TE = "time_text_embed.timestep_embedder."


@pytest.fixture(scope="module")
def env():
    import torch
    from redline_tiny_b200 import _lib as L
    assert torch.cuda.is_available()
    return torch, L, torch.device("cuda:0")


@pytest.fixture(scope="module")
def golden():
    import pathlib
    return dict(np.load(pathlib.Path(__file__).parent / "golden" / "golden.npz"))


def _gpu_glue(env, w, sigma):
    torch, L, dev = env
    s = torch.cuda.current_stream().cuda_stream
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
    l1w, l1b, l2w, l2b = f(w[TE + "linear_1.weight"]), f(w[TE + "linear_1.bias"]), f(w[TE + "linear_2.weight"]), \
        f(w[TE + "linear_2.bias"])
    mw, nw = f(w["modulation.1.weight"]), f(w["norm_out.linear.weight"])
    T = l1w.shape[0]
    freqs = f(HG.timestep_freqs())
    e = torch.empty(2, 256, dtype=torch.float32, device=dev)
    h, te = (torch.empty(2, T, dtype=torch.float32, device=dev) for _ in range(2))
    mod = torch.empty(2, mw.shape[0], dtype=torch.float32, device=dev)
    out = torch.empty(2, nw.shape[0], dtype=torch.float32, device=dev)
    t0 = float(np.float32(HG.model_t(sigma)) * np.float32(1000.0))
    L.call("rl_sinusoidal_embed", t0, 0.0, freqs.data_ptr(), 128, e.data_ptr(), s)
    L.call("rl_matvec_f32", l1w.data_ptr(), T, 256, e.data_ptr(), 2, l1b.data_ptr(), 0, h.data_ptr(), s)
    L.call("rl_matvec_f32", l2w.data_ptr(), T, T, h.data_ptr(), 2, l2b.data_ptr(), 1, te.data_ptr(), s)
    L.call("rl_matvec_f32", mw.data_ptr(), mw.shape[0], T, te.data_ptr(), 2, None, 1, mod.data_ptr(), s)
    L.call("rl_matvec_f32", nw.data_ptr(), nw.shape[0], T, te.data_ptr(), 2, None, 1, out.data_ptr(), s)
    torch.cuda.synchronize()
    return te, mod, out


def test_timestep_embedding_and_modulation_golden(env, golden):
    w = {k[4:]: v for k, v in golden.items() if k.startswith("hw::")}
    te, mod, out = _gpu_glue(env, w, 0.5)
    for got, name in ((te, "temb_05"), (mod, "mod_05"), (out, "normout_05")):
        ref = golden[name]
        assert np.allclose(got.cpu().numpy(), ref, rtol=1e-5, atol=1e-6 * np.abs(ref).max()), name


def test_adaln_params_match_host_rows(env, golden):
    torch, L, dev = env
    w = {k[4:]: v for k, v in golden.items() if k.startswith("hw::")}
    _, mod, out = _gpu_glue(env, w, 0.5)
    D = mod.shape[1] // 4
    params = {k: torch.empty(2, 2, D, dtype=torch.bfloat16, device=dev) for k in ("first", "mlp", "attn", "out")}
    L.call("rl_adaln_params", mod.data_ptr(), out.data_ptr(), out.shape[1], D, params["first"].data_ptr(),
           params["mlp"].data_ptr(), params["attn"].data_ptr(), params["out"].data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = HO.adaln_params(golden["mod_05"], golden["normout_05"], D)
    for k, p in params.items():
        got = p.view(torch.int16).cpu().numpy().astype(np.int32) & 0xFFFF
        want = torch.from_numpy(ref[k]).to(torch.bfloat16).view(torch.int16).numpy().astype(np.int32) & 0xFFFF
        ulps = np.abs(got - want)   # same-sign neighbours differ by one in the bit pattern
        assert ulps.max() <= 1 and (ulps == 0).mean() >= 0.95, (k, ulps.max(), (ulps == 0).mean())


def test_matvec_rows_and_bias(env):
    torch, L, dev = env
    rng = np.random.default_rng(3)
    for N, K, R, silu in ((300, 1028, 3, 1), (8, 12, 4, 0), (1, 4, 1, 1)):
        w = rng.standard_normal((N, K)).astype(np.float32)
        x = rng.standard_normal((R, K)).astype(np.float32)
        b = rng.standard_normal(N).astype(np.float32)
        y = torch.empty(R, N, dtype=torch.float32, device=dev)
        wd, xd, bd = (torch.from_numpy(a).to(dev) for a in (w, x, b))   # held until the kernel has run
        L.call("rl_matvec_f32", wd.data_ptr(), N, K, xd.data_ptr(), R, bd.data_ptr(), silu, y.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        xa = x.astype(np.float64)
        xa = xa / (1 + np.exp(-xa)) if silu else xa
        ref = xa @ w.T.astype(np.float64) + b
        assert np.allclose(y.cpu().numpy(), ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    with pytest.raises(L.RedlineError):
        L.call("rl_matvec_f32", y.data_ptr(), 4, 6, y.data_ptr(), 1, None, 0, y.data_ptr(), 0)    # K % 4 != 0
