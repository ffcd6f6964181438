"""The reference's own DiT host code on the drop-in surface, on CPU: redline/forward.py imported unmodified with
`aie.iron` replaced by redline_tiny_b200.iron (buffers kept in host memory here) and the NPU runtime modules stubbed.
CachedStep (forward.py:209-269) allocates its buffers through the stand-in, and its block loop `blocks`
(forward.py:240-254), `embed` (256-259) and `project` (261-269) run against a recording device; every call must be
one that npu.Device.run maps onto the B200 kernels, with buffers whose sizes Device derives its shapes from
(the GEMM / up+SwiGLU operands, the LayerNorm rows, the QKV-post tables, the attention tiles).

This needs the reference checkout, which exists only where the fixtures are made; the GPU runs of each artifact
family are tests/test_gpu_device.py and tests/test_gpu_npu_formats.py."""

import os
import sys
import types

import numpy as np
import pytest

# the reference checkout's redline/ directory: REDLINE_REFERENCE names the checkout (as make_golden.py's argument
# does); without it the test looks beside this repository
REF = os.path.join(os.environ.get("REDLINE_REFERENCE",
                                  os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "reference")),
                   "redline")


def _forward_module():
    if not os.path.isdir(REF):
        pytest.skip("the reference checkout is not here")
    from redline_tiny_b200 import iron

    class _Any:
        def __init__(self, *a, **k):
            pass

        def __getattr__(self, name):
            return _Any()

        def __call__(self, *a, **k):
            return _Any()

    for name in ("aie", "aie.utils", "aie.utils.npukernel", "aie.utils.trace", "aie.utils.trace.utils", "pyxrt"):
        m = types.ModuleType(name)
        m.__getattr__ = lambda attr: _Any()
        sys.modules[name] = m
    sys.modules["aie.utils"].DefaultNPURuntime = _Any()
    sys.modules["aie.utils.npukernel"].NPUKernel = _Any
    sys.modules["aie.iron"] = iron
    sys.modules["aie"].iron = iron
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import forward
    return forward


class Recorder:
    """Records forward.py's device calls and checks each against npu.Device's artifact map and size rules."""

    def __init__(self):
        from redline_tiny_b200 import npu
        self.npu = npu
        self.calls = []

    def run(self, op, art, args):
        from redline_tiny_b200.iron import Tensor
        assert all(isinstance(a, Tensor) for a in args), f"{art}: a buffer that is not an iron tensor"
        nb = [a.nbytes for a in args]
        if art.startswith(("atb3sw", "vlm-upsw")):
            M, K, N2 = self.npu.Device._mkn(*(_Bytes(n) for n in nb), c_scale=2)
            assert N2 % 256 == 0
        elif art.startswith(("atb3", "q-atb3", "vlm-gemm")):
            self.npu.Device._mkn(*(_Bytes(n) for n in nb))
        elif art.startswith("glue-ln"):
            x, br, p, xo, a = args
            D = p.nbytes // 2 // 4
            assert x.nbytes == xo.nbytes and br.nbytes == a.nbytes == x.nbytes // 2 * 9 // 8 and D * 4 * 2 == p.nbytes
        elif art.startswith("glue-qkv"):
            c, tabs, q, kv = args
            T = tabs.nbytes // 2 // self.npu.TAB_ROW
            assert kv.nbytes == 2 * q.nbytes and q.nbytes % (T * self.npu.TILE_BYTES) == 0
        elif art.startswith(("attn32o", "attn32q")):
            assert len(args) in (3, 4)
        else:
            raise AssertionError(f"artifact {art!r} is not mapped by npu.Device")
        self.calls.append((op, art))

    def sync(self):
        pass


class _Bytes:
    """A stand-in with the numel() of a uint8 buffer of n bytes (Device._mkn reads only sizes)."""

    def __init__(self, n):
        self.n = n

    def numel(self):
        return self.n


def test_cached_step_block_loop_runs_on_the_dropin_surface():
    fw = _forward_module()
    from redline_tiny_b200 import iron
    iron.set_device("cpu")
    try:
        HID, FF, M = fw.HID, fw.FF, 4096
        V9 = fw.V9

        def packed(K, N):
            return iron.tensor(np.zeros(K * N // 8, V9), dtype=V9, device="npu")

        class W:
            pass
        w = W()
        w.b = {}
        rng = np.random.default_rng(0)
        for i in range(2):
            for op, (K, N) in (("qkv", (HID, 3 * HID)), ("o", (HID, HID)), ("up", (HID, 2 * FF)),
                               ("down", (FF, HID))):
                w.b[i, op] = packed(K, N)
            w.b[i, "norm_q"] = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
            w.b[i, "norm_k"] = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
        w.b["img_in"], w.b["proj_out"] = packed(64, HID), packed(HID, 1024)
        ang = rng.uniform(-np.pi, np.pi, (M, 64))
        cs = fw.CachedStep(w, np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32), None)
        cs.attn = lambda n, q, kvt, kvp, o: n.run("attn", fw.ATTN_TARGET, [q, kvt, kvp, o])
        mod = (0.1 * rng.standard_normal((2, 4 * HID))).astype(np.float32)
        cs.set_t(mod, (0.1 * rng.standard_normal((2, HID))).astype(np.float32))
        dev = Recorder()
        lat = iron.tensor(np.zeros(M * 64 // 8, V9), dtype=V9, device="npu")
        cs.embed(dev, lat)
        kv_prefix = {i: iron.zeros((32 * 65 * 2 * 64 * 128 // 8,), dtype=V9, device="npu") for i in range(2)}
        assert cs.blocks(dev, kv_prefix, 0, 1) == 0
        v = cs.project(dev)
        assert v.shape == (M, 64)
    finally:
        iron.set_device(None)
    ops = [c[0] for c in dev.calls]
    per_block = ["qkv", "qkv_post", "attn", "o", "ln_mod", "up_swiglu", "down", "ln_mod"]
    assert ops == ["img_in", "ln_mod"] + per_block * 2 + ["proj_out"], ops


def test_iron_views_and_mutate_on_host():
    """subview offsets are bytes into the parent buffer; mutate writes the host copy back."""
    from redline_tiny_b200 import iron
    iron.set_device("cpu")
    try:
        V9 = np.dtype("V9")
        t = iron.zeros((64,), dtype=V9)
        sub = t.subview(9 * 10, (4,), V9)
        with sub.mutate() as arr:
            arr.view(np.uint8)[:] = np.arange(36, dtype=np.uint8)
        raw = t.numpy().view(np.uint8).reshape(-1)
        assert np.array_equal(raw[90:126], np.arange(36)) and not raw[:90].any() and not raw[126:].any()
        f = iron.tensor(np.arange(6, dtype=np.float32).reshape(2, 3))
        assert f.torch().dtype.__str__() == "torch.float32" and np.array_equal(f.numpy(), np.arange(6).reshape(2, 3))
        with pytest.raises(ValueError):
            t.subview(9 * 63, (2,), V9)
    finally:
        iron.set_device(None)
