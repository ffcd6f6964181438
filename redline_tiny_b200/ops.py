"""Row-major PyTorch-facing API of the bfp16 hot path (torch CUDA tensors in, torch CUDA tensors out).

torch provides device memory and streams only; every computation is a CUDA kernel of libredline_b200.so, called
through its C ABI on the current torch stream.

  quantize_bfp16   npu_layouts.to_bfp16 (+ a_layout)             redline/npu_layouts.py:62-88, 18-23
  dequantize_bfp16 npu_layouts.from_bfp16 (+ a_unlayout)          redline/npu_layouts.py:90-94, 56-60
  pack_b           pack_weights.pack_b                            redline/pack_weights.py:72-79
  PackedWeight     a packed B operand resident on the GPU (native tile order)
  linear_bfp16     gemm() / matmul_vectorized_bfp16 (+ bias)      redline/forward.py:194-197
  swiglu_up        matmul_swiglu_bfp16 (up GEMM + SwiGLU flush)   kernels/atb3/mm_bfp_swiglu.cc:88-168
"""

import torch

from . import _lib as L


def _stream():
    return ctypes_ptr(torch.cuda.current_stream().cuda_stream)


def ctypes_ptr(v):
    return None if v is None else int(v)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _check_cuda(*ts):
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise ValueError("redline_tiny_b200 ops take CUDA tensors (no CPU path)")
            if not t.is_contiguous():
                raise ValueError("tensor must be contiguous")


def _dtype_code(t):
    if t.dtype == torch.float32:
        return L.RL_F32
    if t.dtype == torch.bfloat16:
        return L.RL_BF16
    raise ValueError(f"unsupported dtype {t.dtype}")


_LAYOUTS = {"rowmajor": L.RL_ROWMAJOR, "a_layout": L.RL_A_LAYOUT, "c_atb": L.RL_C_ATB}


def permute_bf16(x, M, K, src="rowmajor", dst="c_atb", out=None):
    """bf16 (M, K) values from one stream order to another (flat tensors for the NPU orders)."""
    _check_cuda(x, out)
    if out is None:
        out = torch.empty(M * K, dtype=torch.bfloat16, device=x.device)
    L.call("rl_permute_bf16", _ptr(x), _LAYOUTS[src], _ptr(out), _LAYOUTS[dst], M, K, _stream())
    return out


def quantize_bfp16(x, layout="rowmajor", want_bytes=True, want_decoded=True):
    """x (M, K) fp32/bf16 -> (bfp16 bytes uint8 [M*K/8*9] in `layout` order or None,
    decoded bf16 (M, K) row-major or None)."""
    _check_cuda(x)
    M, K = x.shape
    q = torch.empty(M * K // 8 * 9, dtype=torch.uint8, device=x.device) if want_bytes else None
    dq = torch.empty((M, K), dtype=torch.bfloat16, device=x.device) if want_decoded else None
    L.call("rl_quantize_bfp16", _ptr(x), _dtype_code(x), M, K, _LAYOUTS[layout], _ptr(q), _ptr(dq), _stream())
    return q, dq


def dequantize_bfp16(q, M, K, layout="rowmajor", dtype=torch.float32):
    _check_cuda(q)
    out = torch.empty((M, K), dtype=dtype, device=q.device)
    L.call("rl_dequantize_bfp16", _ptr(q), _LAYOUTS[layout], M, K, _ptr(out), _dtype_code(out), _stream())
    return out


def pack_b(B):
    """B (K, N) fp32/bf16 -> the reference's packed stream to_bfp16(b_layout(B, 64, 128)) as uint8."""
    _check_cuda(B)
    K, N = B.shape
    out = torch.empty(K * N // 8 * 9, dtype=torch.uint8, device=B.device)
    L.call("rl_pack_b", _ptr(B), _dtype_code(B), K, N, _ptr(out), _stream())
    return out


class PackedWeight:
    """A B operand (K, N) resident on the GPU in the native tile order (1.125 bytes per weight).

    swiglu=True marks an up matrix with [gate 64 | proj 64] per 128 columns (pack_weights.interleave_up); its
    rows are arranged for the fused SwiGLU epilogue."""

    def __init__(self, native, K, N, swiglu=False):
        self.native, self.K, self.N, self.swiglu = native, int(K), int(N), bool(swiglu)

    @classmethod
    def from_pack_b(cls, packed, K, N, swiglu=False):
        """The reference's packed bytes (bNN_*.bin contents, as a CUDA uint8 tensor) -> native tiles."""
        _check_cuda(packed)
        if packed.numel() != K * N // 8 * 9:
            raise ValueError(f"packed stream has {packed.numel()} bytes, expected {K * N // 8 * 9}")
        native = torch.empty_like(packed)
        L.call("rl_weights_from_pack_b", _ptr(packed), K, N, int(swiglu), _ptr(native), _stream())
        return cls(native, K, N, swiglu)

    @classmethod
    def from_float(cls, B, swiglu=False):
        """Float B (K, N) on the GPU -> native tiles (quantised on the device)."""
        _check_cuda(B)
        K, N = B.shape
        native = torch.empty(K * N // 8 * 9, dtype=torch.uint8, device=B.device)
        L.call("rl_pack_weights", _ptr(B), _dtype_code(B), K, N, int(swiglu), _ptr(native), _stream())
        return cls(native, K, N, swiglu)

    def shard(self, rank, world):
        """Columns [n0, n0 + N / world) of this weight as a view of its own bytes (no copy): the N-split standalone
        GEMM's operand on GPU `rank`. Returns (PackedWeight, n0)."""
        n0, cols, off, count = weights_shard(self.K, self.N, rank, world)
        return PackedWeight(self.native.narrow(0, off, count), self.K, cols, self.swiglu), n0


def weights_shard(K, N, rank, world):
    """(n0, n_cols, byte_offset, byte_count) of column shard `rank` of `world` of a packed B (K, N): the same bytes
    in the reference's pack_b stream and in the native tiles (rl_weights_shard)."""
    import ctypes
    v = [ctypes.c_int64() for _ in range(4)]
    L.call("rl_weights_shard", int(K), int(N), int(rank), int(world), *[ctypes.byref(x) for x in v])
    return tuple(x.value for x in v)


def gemm_workspace(M, K, N, device, workspace=None, epilogue=L.RL_EPI_NONE):
    """A device workspace for the GEMM's split-K schedule (rl_linear_bfp16_workspace bytes; None when the shape does
    not split). A given workspace that is large enough is reused."""
    need = L.lib().rl_linear_bfp16_workspace(int(M), int(K), int(N), int(epilogue))
    if need == 0:
        return None
    if workspace is not None and workspace.numel() >= need:
        return workspace
    return torch.empty(need, dtype=torch.uint8, device=device)


def linear_bfp16(x_dq, w, bias=None, out=None, out_dtype=torch.bfloat16, workspace=None):
    """C = x_dq @ B (+ bias), x_dq = bf16 (M, K) holding bfp16 values (quantize_bfp16's decoded output). Shapes with
    too few tiles to fill the GPU and a long K run split-K through a workspace (`workspace`, else one from torch's
    allocator)."""
    _check_cuda(x_dq, w.native, bias, out, workspace)
    if x_dq.dtype != torch.bfloat16:
        raise ValueError("x must be bf16 holding bfp16-exact values (quantize_bfp16 decoded output)")
    M, K = x_dq.shape
    if K != w.K:
        raise ValueError(f"K mismatch: x has {K}, weight has {w.K}")
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=x_dq.device)
    epi = L.RL_EPI_BIAS if bias is not None else L.RL_EPI_NONE
    ws = gemm_workspace(M, K, w.N, x_dq.device, workspace, epi)
    L.call("rl_linear_bfp16_ws", _ptr(x_dq), M, K, _ptr(w.native), w.N, _ptr(bias), epi, _ptr(out),
           _dtype_code(out), _ptr(ws), 0 if ws is None else ws.numel(), _stream())
    return out


def swiglu_up(x_dq, w_up, bias=None, out=None):
    """H = silu(x @ Bgate) * (x @ Bproj), rounded to bfp16 blocks of 8 along F and returned as bf16 (M, F): the
    down projection's A operand. w_up must be packed with swiglu=True."""
    _check_cuda(x_dq, w_up.native, bias, out)
    if not w_up.swiglu:
        raise ValueError("swiglu_up needs a PackedWeight packed with swiglu=True")
    M, K = x_dq.shape
    if out is None:
        out = torch.empty((M, w_up.N // 2), dtype=torch.bfloat16, device=x_dq.device)
    L.call("rl_linear_bfp16", _ptr(x_dq), M, K, _ptr(w_up.native), w_up.N, _ptr(bias), L.RL_EPI_SWIGLU,
           _ptr(out), L.RL_BF16, _stream())
    return out


def swiglu_mlp(x, w_up, w_down, out=None, out_dtype=torch.bfloat16, x_quantized=False, workspace=None):
    """out = (silu(x @ Bgate) * (x @ Bproj)) @ Bdown with bfp16 operands (H rounded to bfp16, as the reference's
    fused flush does). x (M, K) bf16/fp32 raw activations (or bf16 bfp16-exact values with x_quantized=True)."""
    _check_cuda(x, w_up.native, w_down.native, out)
    if not w_up.swiglu:
        raise ValueError("w_up must be packed with swiglu=True")
    M, K = x.shape
    F = w_up.N // 2
    if w_down.K != F or w_up.K != K:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, up ({w_up.K}, {w_up.N}), down ({w_down.K}, {w_down.N})")
    if out is None:
        out = torch.empty((M, w_down.N), dtype=out_dtype, device=x.device)
    need = L.lib().rl_swiglu_mlp_workspace(M, K, F, int(x_quantized))
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    L.call("rl_swiglu_mlp", _ptr(x), _dtype_code(x), int(x_quantized), M, K, _ptr(w_up.native), w_up.N,
           _ptr(w_down.native), w_down.N, _ptr(out), _dtype_code(out), _ptr(workspace), workspace.numel(), _stream())
    return out


def ln_mod(x, branch, params, row_split=0, want_x=True, want_y_bytes=False, rms=False):
    """x' = bf16(x + g * branch); y = LayerNorm(x') * sc (rms=True: RMSNorm, vlm_run.rms_ref) rounded to bfp16
    (run_ln.ln_ref). params: bf16 (2, 2, D) = two rows [g | sc] (run_ln.ln_params); rows < row_split use row 1.
    Returns (x' bf16 or None, y decoded bf16, y bfp16 bytes or None)."""
    _check_cuda(x, branch, params)
    M, D = x.shape
    xo = torch.empty_like(x) if want_x else None
    y = torch.empty_like(x)
    yq = torch.empty(M * D // 8 * 9, dtype=torch.uint8, device=x.device) if want_y_bytes else None
    bdt = L.RL_BF16 if branch is None else _dtype_code(branch)
    L.call("rl_rms_mod" if rms else "rl_ln_mod", _ptr(x), _ptr(branch), bdt, _ptr(params), M, D, int(row_split),
           _ptr(xo), _ptr(y), _ptr(yq), _stream())
    return xo, y, yq


def qkv_post(qkv, rope_cs, w_q, w_k, heads, ldv=None, kv_heads=None):
    """QKV GEMM output (M, (H + 2 Hkv) * 128) -> q (H, M, 128), k (Hkv, M, 128) after RMSNorm * w and RoPE;
    vt (Hkv, 128, ldv) = V^T. kv_heads defaults to heads (no grouping)."""
    _check_cuda(qkv, rope_cs, w_q, w_k)
    M = qkv.shape[0]
    hkv = heads if kv_heads is None else int(kv_heads)
    ldv = ldv or (M + 127) // 128 * 128
    q = torch.empty((heads, M, 128), dtype=torch.bfloat16, device=qkv.device)
    k = torch.empty((hkv, M, 128), dtype=torch.bfloat16, device=qkv.device)
    vt = torch.empty((hkv, 128, ldv), dtype=torch.bfloat16, device=qkv.device)
    L.call("rl_qkv_post_gqa", _ptr(qkv), _ptr(rope_cs), _ptr(w_q), _ptr(w_k), M, heads, hkv, _ptr(q), _ptr(k),
           _ptr(vt), ldv, _stream())
    return q, k, vt


def qkv_linear(x_dq, w, rope_cs, w_q, w_k, heads, ldv=None, kv_heads=None):
    """linear_bfp16(x_dq, w) followed by qkv_post in one GEMM launch (the norm and RoPE run in the GEMM's epilogue):
    w = the packed (K, (H + 2 Hkv) * 128) QKV weight. Outputs as qkv_post."""
    _check_cuda(x_dq, w.native, rope_cs, w_q, w_k)
    M, K = x_dq.shape
    hkv = heads if kv_heads is None else int(kv_heads)
    if w.N != (heads + 2 * hkv) * 128:
        raise ValueError(f"qkv_linear: weight has {w.N} columns, heads need {(heads + 2 * hkv) * 128}")
    ldv = ldv or (M + 127) // 128 * 128
    q = torch.empty((heads, M, 128), dtype=torch.bfloat16, device=x_dq.device)
    k = torch.empty((hkv, M, 128), dtype=torch.bfloat16, device=x_dq.device)
    vt = torch.empty((hkv, 128, ldv), dtype=torch.bfloat16, device=x_dq.device)
    L.call("rl_qkv_linear", _ptr(x_dq), M, K, _ptr(w.native), heads, hkv, _ptr(rope_cs), _ptr(w_q), _ptr(w_k),
           _ptr(q), _ptr(k), _ptr(vt), ldv, _stream())
    return q, k, vt


def attention(q, k, vt, nkv=None, row_limit=None, scale_log2=None, out=None, ldo=None, out_dtype=torch.bfloat16):
    """Flash attention per head: q (H, Nq, 128), k (Hkv, Nk, 128), vt (Hkv, 128, ldv) bf16 -> o (Nq, ldo) with
    head h at columns 128h..; bf16 rounded to bfp16 along the head dim (the out-projection's A operand), or with
    out_dtype=torch.float32 the unrounded fp32 O / l. With Hkv < H query head h reads K/V head h / (H / Hkv)
    (grouped-query attention). scale_log2 defaults to log2(e)/sqrt(128)."""
    import math
    _check_cuda(q, k, vt, row_limit, out)
    H, Nq, _ = q.shape
    Nk = k.shape[1]
    ldv = vt.shape[2]
    nkv = Nk if nkv is None else int(nkv)
    scale_log2 = math.log2(math.e) / math.sqrt(128) if scale_log2 is None else float(scale_log2)
    ldo = ldo or H * 128
    if out is None:
        out = torch.empty((Nq, ldo), dtype=out_dtype, device=q.device)
    if row_limit is not None and row_limit.dtype != torch.int32:
        raise ValueError("row_limit must be int32")
    fn = "rl_attention_gqa_f32" if out.dtype == torch.float32 else "rl_attention_gqa"
    L.call(fn, _ptr(q), _ptr(k), _ptr(vt), ldv, H, k.shape[0], Nq, Nk, nkv, _ptr(row_limit), scale_log2, _ptr(out),
           ldo, _stream())
    return out


def conv_k(cin, taps):
    """The conv GEMM's K: taps^2 taps of Cin channels, each rounded up to a multiple of 64 (zero rows)."""
    return taps * taps * ((cin + 63) // 64 * 64)


def conv_weight(w, bias=None, cout_pad=128):
    """Conv weight (Cout, Cin, k, k), k = 3 or 1, on the GPU -> (PackedWeight of B = [(dy, dx, ci)][co], bf16 bias or
    None, taps). Each tap's Cin rows are zero-padded to a multiple of 64 (K = conv_k(Cin, k)), Cout to a multiple of
    `cout_pad` (the GEMM's N tile)."""
    _check_cuda(w, bias)
    cout, cin, k, _ = w.shape
    n = (cout + cout_pad - 1) // cout_pad * cout_pad
    kt = conv_k(cin, 1)
    B = torch.zeros((k * k, kt, n), dtype=torch.float32, device=w.device)
    B[:, :cin, :cout] = w.float().permute(2, 3, 1, 0).reshape(k * k, cin, cout)
    B = B.reshape(k * k * kt, n)
    b = None
    if bias is not None:
        b = torch.zeros(n, dtype=torch.bfloat16, device=w.device)
        b[:cout] = bias.to(torch.bfloat16)
    return PackedWeight.from_float(B), b, k


def conv2d(x_dq, w, bias, taps, out=None):
    """VAE conv: x_dq (H, W, Cin) bf16 holding bfp16 values -> (H, W, N) bf16 (N = the padded Cout)."""
    _check_cuda(x_dq, w.native, bias, out)
    H, Wd, C = x_dq.shape
    if w.K != conv_k(C, taps):
        raise ValueError(f"conv weight has K = {w.K}, a {taps}x{taps} conv over {C} channels needs {conv_k(C, taps)}")
    if out is None:
        out = torch.empty((H, Wd, w.N), dtype=torch.bfloat16, device=x_dq.device)
    nbytes = L.lib().rl_conv2d_workspace(H, Wd, C, taps)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x_dq.device)
    L.call("rl_conv2d_bfp16", _ptr(x_dq), H, Wd, C, _ptr(w.native), w.N, taps, _ptr(bias), _ptr(out), _ptr(ws),
           ws.numel(), _stream())
    return out


def set_gemm_variant(v):
    return L.lib().rl_set_gemm_variant(int(v))


def set_attention_variant(v):
    """0 = two query tiles per CTA (default), 1 = one query tile per CTA; returns the previous choice."""
    return L.lib().rl_set_attention_variant(int(v))


def device_status():
    return L.device_status()
