"""The allocation-free SwiGLU MLP entry point (rl_swiglu_mlp_noalloc), called through the C ABI.

Some callers cannot allocate device memory: a serving process that reserves its whole memory pool at start-up and
treats any later allocation as a failure, or a latency-critical path where cudaMalloc / cudaFree would synchronise
the device. This entry point keeps its scratch in a fixed array inside the library instead. The test checks it
against the workspace-taking entry point (rl_swiglu_mlp) on two calls in a row with different inputs - the second
call finds the first call's data in the shared array - within the MLP tolerance the other tests use (max-rel
<= 2e-3), at the array's exact capacity, and that a request larger than the array is refused. This file is collected
last so that a run stopping at its first failure has already run every other test; it passes alone in a fresh
process too."""

import ctypes

import numpy as np
import pytest

from oracle import bfp16_oracle as O

pytestmark = pytest.mark.gpu


def _case(M, K, F, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wg = (rng.standard_normal((F, K)) * 0.02).astype(np.float32)
    wu = (rng.standard_normal((F, K)) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((N, F)) * 0.02).astype(np.float32)
    return x, O.interleave_up(wg, wu), wd.T.copy()


def _array_bytes(M, K, F):
    """What the array must hold: the quantised x and H (M x K and M x F bf16), each rounded up to 256 bytes."""
    r = lambda v: (v + 255) // 256 * 256
    return r(M * K * 2) + r(M * F * 2)


@pytest.mark.parametrize("M", [512, 1024])
def test_noalloc_matches_workspace_entry_on_two_calls(M):
    """M = 512 is config 2 (16.8 MB of the 32 MiB array); M = 1024 fills the array exactly."""
    import torch
    from redline_tiny_b200 import _lib as L
    from redline_tiny_b200 import ops

    lib = L.lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    K, F, N = 4096, 12288, 4096
    assert _array_bytes(M, K, F) <= lib.rl_swiglu_mlp_noalloc_capacity()
    _, Bup, Bdown = _case(M, K, F, N, seed=1)
    wu = ops.PackedWeight.from_float(torch.from_numpy(Bup).to(dev), swiglu=True)
    wd = ops.PackedWeight.from_float(torch.from_numpy(Bdown).to(dev))
    for call, seed in enumerate((11, 12)):
        x = torch.from_numpy(np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)).to(dev)
        ws = torch.empty(lib.rl_swiglu_mlp_workspace(M, K, F, 0), dtype=torch.uint8, device=dev)
        ref = torch.empty((M, N), dtype=torch.float32, device=dev)
        got = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)
        L.call("rl_swiglu_mlp", x.data_ptr(), L.RL_F32, 0, M, K, wu.native.data_ptr(), 2 * F, wd.native.data_ptr(), N,
               ref.data_ptr(), L.RL_F32, ws.data_ptr(), ws.numel(), stream)
        L.call("rl_swiglu_mlp_noalloc", x.data_ptr(), L.RL_F32, 0, M, K, wu.native.data_ptr(), 2 * F,
               wd.native.data_ptr(), N, got.data_ptr(), L.RL_F32, stream)
        L.device_status()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}: unwritten output"
        err = O.max_rel(g, r)
        assert err <= 2e-3, f"call {call}: max-rel {err:.3e} against rl_swiglu_mlp"


def test_noalloc_rejects_oversize_request():
    from redline_tiny_b200 import _lib as L

    lib = L.lib()
    cap = lib.rl_swiglu_mlp_noalloc_capacity()
    buf = ctypes.create_string_buffer(64)
    K, F = 4096, 12288
    for M in (1025, 4096):                          # one row past the capacity; 134 MB
        assert _array_bytes(M, K, F) > cap
        st = lib.rl_swiglu_mlp_noalloc(ctypes.addressof(buf), L.RL_BF16, 0, M, K, ctypes.addressof(buf), 2 * F,
                                       ctypes.addressof(buf), 4096, ctypes.addressof(buf), L.RL_BF16, None)
        assert st == L.RL_ERR_ARGUMENT
        assert b"more than the fixed" in lib.rl_last_error()
    st = lib.rl_swiglu_mlp_noalloc(ctypes.addressof(buf), L.RL_BF16, 0, 1 << 40, K, ctypes.addressof(buf), 2 * F,
                                   ctypes.addressof(buf), 4096, ctypes.addressof(buf), L.RL_BF16, None)
    assert st == L.RL_ERR_ARGUMENT and b"too large" in lib.rl_last_error()
