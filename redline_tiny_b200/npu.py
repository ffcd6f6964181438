"""Drop-in for the reference's device object: `Device.run(op, artifact, args)` with the reference's own buffers.

The reference's DiT and text encoder call every kernel as `npu.run(op, artifact_name, [iron tensors])`
(redline/forward.py:138-165; vlm_run.py:56-57). `Device` keeps that contract on a B200: `args` are torch CUDA tensors
holding the same bytes as the reference's buffers - bfp16 blocks (uint8, 9 bytes per 8 values) in the NPU stream
orders (a_layout A operands, pack_b weights, ATB-order C), bf16 residual streams in the ATB C order - and each
artifact family maps onto the B200 kernels through the C ABI:

  GEMM ("atb3d2-*", "q-atb3k-*", "vlm-gemm-*")  [A, B, C]       forward.py:194-197  (C in ATB order, bfp16)
  up + SwiGLU ("atb3sw2-*", "vlm-upsw*")        [A, B_up, H]    forward.py:250      (H as the down GEMM's A)
  ln_mod ("glue-ln-m{M}-s{S}")                  [x, br, p, x', A]  forward.py:249    (rows < 128 S use row 1)

Shapes come from the buffer sizes (the reference fixes them per artifact). Packed weights are repacked once into the
native tile format and cached per weight buffer, like the reference's resident `Weights` (forward.py:175-191). The
QKV-post and attention artifacts use NPU-specific tile orders (per-64-token Q / K / V tiles, kernels/glue/qkv_post.cc,
kernels/attn/attn_bfp.cc) and are not mapped: on B200 the DiT runs through redline_tiny_b200.dit, which keeps Q, K, V
in row-major head-major buffers.
"""

import math
import re
import time
from collections import defaultdict

import torch

from . import _lib as L
from . import ops


class Device:
    """Stand-in for forward.NPU: run / sync / report with per-op wall time and call counts."""

    def __init__(self):
        self.t_wall, self.calls = defaultdict(float), defaultdict(int)
        self._native = {}

    # -- the reference's interface --------------------------------------------------------------------------------
    def run(self, op, art, args):
        t = time.perf_counter()
        if art.startswith(("atb3sw", "vlm-upsw")):
            self._up_swiglu(*args)
        elif art.startswith(("atb3", "q-atb3", "vlm-gemm")):
            self._gemm(*args)
        elif art.startswith("glue-ln"):
            m = re.search(r"-s(\d+)", art)
            self._ln_mod(*args, row_split=128 * int(m.group(1)) if m else 0)
        else:
            raise NotImplementedError(
                f"artifact {art!r}: the NPU's QKV-post / attention tile formats are not mapped; run the DiT with "
                "redline_tiny_b200.dit on B200")
        self.t_wall[op] += time.perf_counter() - t
        self.calls[op] += 1

    def sync(self):
        torch.cuda.synchronize()

    def report(self):
        for op in sorted(self.t_wall, key=lambda o: -self.t_wall[o]):
            print(f"  {op:12s} {self.calls[op]:5d} calls  wall {self.t_wall[op] * 1e3:9.1f} ms")

    # -- artifact families ------------------------------------------------------------------------------------------
    def _weight(self, b, K, N, swiglu=False):
        key = (b.data_ptr(), b.numel(), swiglu)
        w = self._native.get(key)
        if w is None:
            w = self._native[key] = ops.PackedWeight.from_pack_b(b.view(torch.uint8).reshape(-1), K, N, swiglu)
        return w

    @staticmethod
    def _mkn(a, b, c, c_scale=1):
        """M, K, N from the bfp16 byte counts of A (M x K), B (K x N) and C (M x N / c_scale)."""
        va, vb, vc = a.numel() * 8 // 9, b.numel() * 8 // 9, c.numel() * 8 // 9 * c_scale
        M = round(math.sqrt(va * vc / vb))
        K, N = va // M, vc // M
        assert M * K == va and K * N == vb and M * N == vc, "buffer sizes do not form a GEMM"
        return M, K, N

    def _gemm(self, a, b, c):
        a, b, c = (t.view(torch.uint8).reshape(-1) for t in (a, b, c))
        M, K, N = self._mkn(a, b, c)
        x = ops.dequantize_bfp16(a, M, K, layout="a_layout", dtype=torch.bfloat16)
        y = ops.linear_bfp16(x, self._weight(b, K, N), out_dtype=torch.float32)
        L.call("rl_quantize_bfp16", y.data_ptr(), L.RL_F32, M, N, L.RL_C_ATB, c.data_ptr(), None,
               torch.cuda.current_stream().cuda_stream)

    def _up_swiglu(self, a, b, h):
        a, b, h = (t.view(torch.uint8).reshape(-1) for t in (a, b, h))
        M, K, N2 = self._mkn(a, b, h, c_scale=2)
        x = ops.dequantize_bfp16(a, M, K, layout="a_layout", dtype=torch.bfloat16)
        hv = ops.swiglu_up(x, self._weight(b, K, N2, swiglu=True))
        L.call("rl_quantize_bfp16", hv.data_ptr(), L.RL_BF16, M, N2 // 2, L.RL_A_LAYOUT, h.data_ptr(), None,
               torch.cuda.current_stream().cuda_stream)

    def _ln_mod(self, x, br, params, xo, a, row_split=0):
        D = params.numel() // 4
        M = x.numel() // D
        s = torch.cuda.current_stream().cuda_stream
        xr = ops.permute_bf16(x.view(torch.bfloat16).reshape(-1), M, D, src="c_atb", dst="rowmajor")
        brr = ops.dequantize_bfp16(br.view(torch.uint8).reshape(-1), M, D, layout="c_atb", dtype=torch.bfloat16)
        x1 = torch.empty(M * D, dtype=torch.bfloat16, device=x.device)
        y = torch.empty(M * D, dtype=torch.bfloat16, device=x.device)
        L.call("rl_ln_mod", xr.data_ptr(), brr.data_ptr(), L.RL_BF16, params.data_ptr(), M, D, row_split,
               x1.data_ptr(), y.data_ptr(), None, s)
        L.call("rl_permute_bf16", x1.data_ptr(), L.RL_ROWMAJOR, xo.data_ptr(), L.RL_C_ATB, M, D, s)
        L.call("rl_quantize_bfp16", y.data_ptr(), L.RL_BF16, M, D, L.RL_A_LAYOUT, a.data_ptr(), None, s)


def gemm(npu, w, op, M, a, c, block=None):
    """forward.gemm (forward.py:194-197) on a Device: `w.b[block, op]` holds the packed B as a CUDA uint8 tensor."""
    b = w.b[block, op] if block is not None else w.b[op]
    npu.run(op, f"atb3-{op}-m{M}", [a, b, c])
