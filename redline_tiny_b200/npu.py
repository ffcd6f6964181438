"""Drop-in for the reference's device object: `Device.run(op, artifact, args)` with the reference's own buffers.

The reference's DiT and text encoder call every kernel as `npu.run(op, artifact_name, [iron tensors])`
(redline/forward.py:138-165; vlm_run.py:56-57). `Device` keeps that contract on a B200: `args` are torch CUDA tensors
holding the same bytes as the reference's buffers - bfp16 blocks (uint8, 9 bytes per 8 values) in the NPU stream
orders (a_layout A operands, pack_b weights, ATB-order C), bf16 residual streams in the ATB C order - and each
artifact family maps onto the B200 kernels through the C ABI:

  GEMM ("atb3d2-*", "q-atb3k-*", "vlm-gemm-*")  [A, B, C]       forward.py:194-197  (C in ATB order, bfp16)
  up + SwiGLU ("atb3sw2-*", "vlm-upsw*")        [A, B_up, H]    forward.py:250      (H as the down GEMM's A)
  ln_mod ("glue-ln-m{M}-s{S}")                  [x, br, p, x', A]  forward.py:249    (rows < 128 S use row 1)
  QKV post ("glue-qkv*")                        [C_qkv, tabs, Q, KV]  forward.py:246 (per-head 64-token tiles)
  attention ("attn32o-*", "attn32q-*")          [Q, KV, (KV_prefix | LIM), O]  forward.py:251, 365-376, 613

Q and KV hold the reference's attention formats (run_attn.py:29-35, 82-92: Q tiles a_layout(., 64, 128), K tiles
b_layout(K^T, 128, 64), V tiles b_layout(V, 64, 128), bfp16); O is the out-projection's A operand. The attention
forms, as forward.py uses them (the artifacts' tile ranges are fixed by their builds; here they follow from the
name and the buffer sizes):
  attn32o-*-s-*-pf-nk{NK}-nkv{NKV}  [Q, KV_t, KV_p, O]  cached steps: every Q tile over [all of KV_t | KV_p tiles
                                                        0 ..], NK keys, the first NKV valid
  attn32o-*-s-*-tr-nk{NK}-nkv{NKV}  [Q, KV, KV_p, O]    step 1 target: Q / KV tiles of the 4096 target rows (from
                                                        row 4224 at M = 8704, 512 at M = 4608) over [those | KV_p 0 ..]
  attn32o-*-a-*-tr-nk{NK}-nkv{NKV}  [Q, KV, O]          reference-image rows: Q tiles 0..63 over KV tiles 0 ..
  attn32q-*-nk{NK}-pt{PT}           [Q, LIM, KV, O]     up to 64 rows per head over KV tiles 0 .. with per-row key
                                                        limits (LIM: int32 at the start of the buffer, run_attn.pack_lim)
Shapes come from the buffer sizes (the reference fixes them per artifact). Packed weights are repacked once into the
native tile format and cached per weight buffer, like the reference's resident `Weights` (forward.py:175-191).
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
        from .iron import Tensor           # buffers of the aie.iron stand-in: their torch views
        args = [a.torch() if isinstance(a, Tensor) else a for a in args]
        if art.startswith(("atb3sw", "vlm-upsw")):
            self._up_swiglu(*args)
        elif art.startswith(("atb3", "q-atb3", "vlm-gemm")):
            self._gemm(*args)
        elif art.startswith("glue-ln"):
            m = re.search(r"-s(\d+)", art)
            self._ln_mod(*args, row_split=128 * int(m.group(1)) if m else 0)
        elif art.startswith("glue-qkv"):
            self._qkv_post(*args)
        elif art.startswith(("attn32o", "attn32q")):
            self._attention(art, args)
        else:
            raise NotImplementedError(f"artifact {art!r} is not mapped onto the B200 kernels")
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

    # -- QKV post and attention in the NPU tile formats ------------------------------------------------------------
    def _qkv_post(self, c_qkv, tabs, q, kv):
        """C_qkv (bfp16, ATB order, M x 3 HID) -> per-head RMSNorm * w, RoPE on adjacent pairs (tables decoded from
        the reference's qkv_tables rows) -> Q / KV in the attention formats (run_qkv.py:41-79)."""
        c, qb, kvb = (t.view(torch.uint8).reshape(-1) for t in (c_qkv, q, kv))
        tb = tabs.view(torch.bfloat16).reshape(-1)
        T = tb.numel() // TAB_ROW
        M = 64 * T
        n3 = c.numel() * 8 // 9 // M
        H = n3 // 3 // 128
        if tb.numel() != T * TAB_ROW or n3 * M * 9 // 8 != c.numel() or n3 != 3 * 128 * H:
            raise ValueError("qkv_post: C_qkv / table sizes do not match")
        if qb.numel() != H * T * TILE_BYTES or kvb.numel() != 2 * H * T * TILE_BYTES:
            raise ValueError(f"qkv_post: Q / KV buffers must hold {H} heads x {T} tiles")
        s = torch.cuda.current_stream().cuda_stream
        dev = c.device
        cdq = ops.dequantize_bfp16(c, M, n3, layout="c_atb", dtype=torch.bfloat16)
        cs = torch.empty(M, 64, 2, dtype=torch.float32, device=dev)
        wq = torch.empty(128, dtype=torch.float32, device=dev)
        wk = torch.empty(128, dtype=torch.float32, device=dev)
        L.call("rl_npu_qkv_tables", tb.data_ptr(), T, cs.data_ptr(), wq.data_ptr(), wk.data_ptr(), s)
        ldv = (M + 127) // 128 * 128
        qq = torch.empty(H, M, 128, dtype=torch.bfloat16, device=dev)
        kk = torch.empty(H, M, 128, dtype=torch.bfloat16, device=dev)
        vt = torch.zeros(H, 128, ldv, dtype=torch.bfloat16, device=dev)
        L.call("rl_qkv_post", cdq.data_ptr(), cs.data_ptr(), wq.data_ptr(), wk.data_ptr(), M, H, qq.data_ptr(),
               kk.data_ptr(), vt.data_ptr(), ldv, s)
        L.call("rl_npu_qkv_pack", qq.data_ptr(), kk.data_ptr(), vt.data_ptr(), ldv, H, T, qb.data_ptr(),
               kvb.data_ptr(), s)

    @staticmethod
    def _tiles(buf, H, per_tile):
        n = buf.numel()
        if n % (H * per_tile):
            raise ValueError(f"buffer of {n} bytes is not {H} heads of whole tiles")
        return n // (H * per_tile)

    def _attention(self, art, args):
        """The attention artifacts (forms in the module docstring): unpack the Q / K / V tiles each form reads, run
        rl_attention_gqa (Q already carries log2(e) / sqrt(128)), write O as the out-projection's bfp16 A operand."""
        s = torch.cuda.current_stream().cuda_stream
        mo = re.match(r"attn32o-v\d+-([sa])-h(\d+)-t\d+-(pf|tr)-nk(\d+)-nkv(\d+)", art)
        mq = re.match(r"attn32q-v\d+-t\d+-nk(\d+)-pt(\d+)", art)
        if mo:
            split, H, mode, NK, NKV = mo.group(1), int(mo.group(2)), mo.group(3), int(mo.group(4)), int(mo.group(5))
        elif mq:
            H, NK, NKV, split, mode = 32, int(mq.group(1)), int(mq.group(1)), "q", "small"
        else:
            raise NotImplementedError(f"attention artifact {art!r}: unknown form")
        bufs = [t.view(torch.uint8).reshape(-1) for t in args]
        if NK % 64 or not 0 < NKV <= NK:
            raise ValueError(f"{art}: NK must be a multiple of 64 and 0 < NKV <= NK")
        row_limit = None
        if split == "s":
            qb, kvt, kvp, ob = bufs
            Tq, Tt, Tp = (self._tiles(b, H, u) for b, u in ((qb, TILE_BYTES), (kvt, 2 * TILE_BYTES),
                                                            (kvp, 2 * TILE_BYTES)))
            if mode == "pf":
                q_rng, kv_rngs = (0, Tq), [(kvt, Tt, 0, Tt)]
                npre = NK // 64 - Tt
            else:
                t0 = {8704: 4224, 4608: 512}.get(64 * Tq)
                if t0 is None:
                    raise ValueError(f"{art}: target rows of a {64 * Tq}-row step-1 layout are not known")
                q_rng, kv_rngs = (t0 // 64, 64), [(kvt, Tt, t0 // 64, 64)]
                npre = NK // 64 - 64
            if npre < 0 or npre > Tp:
                raise ValueError(f"{art}: {npre} prefix tiles outside the {Tp}-tile prefix buffer")
            if npre:
                kv_rngs.append((kvp, Tp, 0, npre))
        elif split == "a":
            qb, kv, ob = bufs
            Tq, Tk = self._tiles(qb, H, TILE_BYTES), self._tiles(kv, H, 2 * TILE_BYTES)
            q_rng, kv_rngs = (0, min(64, Tq)), [(kv, Tk, 0, NK // 64)]
        else:
            qb, lim, kv, ob = bufs
            Tq, Tk = self._tiles(qb, H, TILE_BYTES), self._tiles(kv, H, 2 * TILE_BYTES)
            if Tk != int(mq.group(2)):
                raise ValueError(f"{art}: the K/V buffer holds {Tk} tiles per head, the artifact reads {mq.group(2)}")
            q_rng, kv_rngs = (0, Tq), [(kv, Tk, 0, NK // 64)]
            row_limit = lim[:4 * 64 * Tq].view(torch.int32)
        dev = bufs[0].device
        nq = 64 * q_rng[1]
        q = torch.empty(H, nq, 128, dtype=torch.bfloat16, device=dev)
        L.call("rl_npu_q_unpack", qb.data_ptr(), H, Tq, q_rng[0], q_rng[1], q.data_ptr(), s)
        k = torch.empty(H, NK, 128, dtype=torch.bfloat16, device=dev)
        vt = torch.empty(H, 128, NK, dtype=torch.bfloat16, device=dev)
        key0 = 0
        for buf, tpl, t0, n in kv_rngs:
            L.call("rl_npu_kv_unpack", buf.data_ptr(), H, tpl, t0, n, key0, NK, NK, k.data_ptr(), vt.data_ptr(), s)
            key0 += 64 * n
        if key0 != NK:
            raise ValueError(f"{art}: the tile ranges give {key0} keys, the artifact reads {NK}")
        rows_out = ob.numel() * 8 // 9 // (H * 128)
        if rows_out * H * 128 * 9 // 8 != ob.numel() or rows_out < nq or rows_out % 128:
            raise ValueError(f"{art}: O must hold a multiple of 128 rows >= {nq} of {H} heads")
        o = torch.zeros(rows_out, H * 128, dtype=torch.bfloat16, device=dev)
        ops.attention(q, k, vt, nkv=NKV, row_limit=row_limit, scale_log2=1.0, out=o[:nq], ldo=H * 128)
        L.call("rl_quantize_bfp16", o.data_ptr(), L.RL_BF16, rows_out, H * 128, L.RL_A_LAYOUT, ob.data_ptr(), None, s)


TILE_BYTES = 64 * 128 // 8 * 9    # one 64-token Q / K / V tile
TAB_ROW = 128 * 64 + 2 * 128      # QKV-post table entries per 64-row tile (run_qkv.TAB)


def gemm(npu, w, op, M, a, c, block=None):
    """forward.gemm (forward.py:194-197) on a Device: `w.b[block, op]` holds the packed B as a CUDA uint8 tensor."""
    b = w.b[block, op] if block is not None else w.b[op]
    npu.run(op, f"atb3-{op}-m{M}", [a, b, c])
