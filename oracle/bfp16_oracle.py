"""CPU oracle for the bfp16 weight-GEMM hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (`redline_tiny_b200`) imports this module; only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of `bench.py` use it, as the checker
and as the timed CPU baseline. It restates, in plain numpy, the reference implementation of the path
(Cukrus-directive/redline-tiny); every function names the reference file:line it follows. Parity of this
restatement is pinned by `tests/golden/*.npz`, which `tests/golden/make_golden.py` generates by importing the
reference's own Python modules and running them on seeded inputs.

bfp16 ("bfp16ebs8"): blocks of 8 consecutive stream values share one 8-bit exponent byte E (the largest biased
float32 exponent field in the block) followed by 8 signed int8 mantissas, 9 bytes per 8 values;
value = mantissa * 2**(E - 133).
"""

import functools

import numpy as np

BLOCK = 8          # values per bfp16 block
BLOCK_BYTES = 9    # [E][m0..m7]
EXP_OFFSET = 133   # value = m * 2**(E - EXP_OFFSET)


# ----------------------------------------------------------------------------------------------------------------
# bf16 rounding (numpy has no bf16; ml_dtypes' cast is round-half-even, which this restates)
# ----------------------------------------------------------------------------------------------------------------

def bf16_round(x):
    """float32 -> nearest bf16 value (round half to even), returned as float32. Finite inputs only."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def bf16_bits(x):
    """float32 values that are already bf16-exact -> their uint16 bf16 bit patterns."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(u16):
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------------------------------------------
# the codec: redline/npu_layouts.py:62-94
# ----------------------------------------------------------------------------------------------------------------

def to_bfp16(x):
    """Stream of float32 values (length a multiple of 8) -> bfp16 bytes. Follows npu_layouts.py:62-88 (the
    round-half-to-even branch): E = the block's largest biased float32 exponent field; m = clip(rint(x * 2**(133-E)),
    -128, 127), with the product formed exactly in float64."""
    v = np.ascontiguousarray(x, np.float32).reshape(-1, BLOCK)
    field = ((v.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    e_blk = field.max(axis=1)
    m = np.rint(v.astype(np.float64) * np.ldexp(1.0, EXP_OFFSET - e_blk)[:, None])
    m = np.clip(m, -128, 127).astype(np.int8)
    out = np.empty((v.shape[0], BLOCK_BYTES), np.uint8)
    out[:, 0] = e_blk.astype(np.uint8)
    out[:, 1:] = m.view(np.uint8)
    return out.reshape(-1)


def to_bfp16_int(x):
    """The same quantiser restated in integer arithmetic, the way the CUDA kernel computes it: the 24-bit significand
    is shifted right by 17 + E - max(e, 1) with round-half-to-even on the dropped bits. Used to show that the
    integer formulation equals the float64 one on every edge case (ties, denormals, saturation)."""
    v = np.ascontiguousarray(x, np.float32).reshape(-1, BLOCK)
    bits = v.view(np.uint32).astype(np.int64)
    field = (bits >> 23) & 0xFF
    e_blk = field.max(axis=1, keepdims=True)
    sig = np.where(field > 0, (bits & 0x7FFFFF) | 0x800000, bits & 0x7FFFFF)
    shift = 17 + e_blk - np.maximum(field, 1)
    big = shift > 25                                     # sig < 2**24, so anything shifted further rounds to 0
    sh = np.minimum(shift, 25)
    q = sig >> sh
    rem = sig & ((np.int64(1) << sh) - 1)
    half = np.int64(1) << (sh - 1)
    q = q + ((rem > half) | ((rem == half) & ((q & 1) == 1))).astype(np.int64)
    q = np.where(big, 0, q)
    m = np.where((bits >> 31) & 1, -q, q)
    m = np.clip(m, -128, 127).astype(np.int8)
    out = np.empty((v.shape[0], BLOCK_BYTES), np.uint8)
    out[:, 0] = e_blk[:, 0].astype(np.uint8)
    out[:, 1:] = m.view(np.uint8)
    return out.reshape(-1)


def from_bfp16(raw):
    """bfp16 bytes -> float64 values m * 2**(E - 133). npu_layouts.py:90-94 (which also yields float64: an int8 ->
    float32 array times a float64 scale). Every such value is exact in bf16 and float32 for E <= 254."""
    blk = np.asarray(raw, np.uint8).reshape(-1, BLOCK_BYTES)
    scale = np.ldexp(1.0, blk[:, 0].astype(np.int64) - EXP_OFFSET)[:, None]
    return (blk[:, 1:].view(np.int8).astype(np.float64) * scale).reshape(-1)


def quantize_rows(x):
    """Row-major (M, K) -> (bfp16 bytes with blocks of 8 along K in row-major order, decoded float32 (M, K))."""
    x = np.ascontiguousarray(x, np.float32)
    q = to_bfp16(x.reshape(-1))
    return q, from_bfp16(q).astype(np.float32).reshape(x.shape)


# ----------------------------------------------------------------------------------------------------------------
# stream layouts: redline/npu_layouts.py:11-60, as explicit index maps (element (r, c) -> stream position)
# ----------------------------------------------------------------------------------------------------------------

@functools.lru_cache(maxsize=8)
def a_layout_index(M, K, m=128, k=64):
    """Stream position of every (r, c) of an (M, K) A operand: npu_layouts.py:18-23 `a_layout` (L1 tiles m x k
    row-major; inside, 16-row bands, then 8-column blocks, then the band's two 8-row halves, then 8x8 row-major).
    Same map as forward.py:74-79 `a_index`."""
    r = np.arange(M)[:, None]
    c = np.arange(K)[None, :]
    tile = (r // m) * (K // k) + c // k
    inner = ((((r % m) // 16) * (k // 8) + (c % k) // 8) * 2 + (r % 16) // 8) * 64 + (r % 8) * 8 + c % 8
    return _frozen(tile * (m * k) + inner)


@functools.lru_cache(maxsize=8)
def b_layout_index(K, N, k=64, n=128):
    """Stream position of every (r, c) of a (K, N) B operand: npu_layouts.py:11-16 `b_layout` (L1 tiles k x n,
    N-tile outer and K-tile inner; inside, 16-column bands, 8-row blocks, the band's two 8-column halves, then
    column-major 8x8: 8 consecutive K of one column are one bfp16 block)."""
    r = np.arange(K)[:, None]
    c = np.arange(N)[None, :]
    tile = (c // n) * (K // k) + r // k
    inner = ((((c % n) // 16) * (k // 8) + (r % k) // 8) * 2 + (c % 16) // 8) * 64 + (c % 8) * 8 + r % 8
    return _frozen(tile * (k * n) + inner)


@functools.lru_cache(maxsize=8)
def c_atb_index(M, N, m=128, n=128, rows=4, cols=8):
    """Stream position of every (r, c) of the (M, N) C the ATB GEMM designs emit: npu_layouts.py:31-48
    `c_layout_atb` (groups of rows x cols tiles, row-group outer; per group one chunk per core column stacking that
    column's `rows` tiles; inside a tile 2x2 super-blocks of row-major 8x8). Same map as forward.py:64-71."""
    r = np.arange(M)[:, None]
    c = np.arange(N)[None, :]
    rg, row, sbr, br, rib = r // (rows * m), (r // m) % rows, (r % m) // 16, (r % 16) // 8, r % 8
    cg, col, sbc, bc, cib = c // (cols * n), (c // n) % cols, (c % n) // 16, (c % 16) // 8, c % 8
    i = (rg * (N // (cols * n)) + cg) * cols + col
    for d, v in ((rows, row), (m // 16, sbr), (n // 16, sbc), (2, br), (2, bc), (8, rib), (8, cib)):
        i = i * d + v
    return _frozen(i)


def _frozen(idx):
    """Index maps are cached per shape (the CPU baseline applies the same maps every step), so they are read-only."""
    idx.setflags(write=False)
    return idx


def _scatter(a, idx):
    a = np.asarray(a)
    out = np.empty(a.size, a.dtype)
    out[idx.reshape(-1)] = a.reshape(-1)
    return out


def _gather(s, idx):
    return np.asarray(s).reshape(-1)[idx]


def a_layout(a, m=128, k=64):
    return _scatter(a, a_layout_index(*np.shape(a), m, k))


def a_unlayout(s, M, K, m=128, k=64):
    return _gather(s, a_layout_index(M, K, m, k))


def b_layout(b, k=64, n=128):
    return _scatter(b, b_layout_index(*np.shape(b), k, n))


def b_unlayout(s, K, N, k=64, n=128):
    return _gather(s, b_layout_index(K, N, k, n))


def c_layout_atb(c, m=128, n=128, rows=4, cols=8):
    return _scatter(c, c_atb_index(*np.shape(c), m, n, rows, cols))


def c_unlayout_atb(s, M, N, m=128, n=128, rows=4, cols=8):
    return _gather(s, c_atb_index(M, N, m, n, rows, cols))


# ----------------------------------------------------------------------------------------------------------------
# packed weights: redline/pack_weights.py:72-89
# ----------------------------------------------------------------------------------------------------------------

def pack_b(B):
    """(K, N) float32 B operand (C = A @ B, so B = W.T) -> the reference's packed weight stream:
    to_bfp16(b_layout(B, 64, 128)). pack_weights.py:72-79."""
    return to_bfp16(b_layout(np.ascontiguousarray(B, np.float32)))


def interleave_up(w_gate, w_proj):
    """gate / proj weights (F, K) -> B (K, 2F) with [gate 64 | proj 64] per 128-column tile. pack_weights.py:82-89."""
    F, K = w_gate.shape
    B = np.empty((K, F // 64, 2, 64), np.float32)
    B[:, :, 0] = np.asarray(w_gate, np.float32).T.reshape(K, F // 64, 64)
    B[:, :, 1] = np.asarray(w_proj, np.float32).T.reshape(K, F // 64, 64)
    return B.reshape(K, 2 * F)


def unpack_b(raw, K, N):
    """Packed stream -> decoded (K, N) float32 B."""
    return b_unlayout(from_bfp16(raw).astype(np.float32), K, N)


# ----------------------------------------------------------------------------------------------------------------
# the ops on the path
# ----------------------------------------------------------------------------------------------------------------

def linear(xd, bd, bias=None):
    """C = A @ B (+ bias) in float32 on already-decoded bfp16 operands: the north-star oracle ("bfp16 packing /
    quantisation followed by an fp32 matmul on the decoded blocks"); forward.py:194-197 `gemm` computes this product
    on the NPU."""
    c = np.asarray(xd, np.float32) @ np.asarray(bd, np.float32)
    if bias is not None:
        c = c + np.asarray(bias, np.float32)[None, :]
    return c


def silu(x):
    """run_glue.py:23-24."""
    return x / (1.0 + np.exp(-x))


def swiglu_from_interleaved(c):
    """(M, 2F) up-GEMM output with [gate 64 | proj 64] per 128 columns -> silu(gate) * proj (M, F).
    The product that mm_bfp_swiglu.cc:73-86 writes (before its bfp16 rounding)."""
    c = np.asarray(c)
    M, N = c.shape
    v = c.reshape(M, N // 128, 2, 64)
    return (silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)


def ln_ref(xq, brq, g, sc):
    """redline/run_ln.py:65-71: x' = bf16(x + bf16(g) * branch) (float32 arithmetic), then LayerNorm of x' in
    float64 (eps 1e-6, no affine) times bf16(sc)."""
    t = np.asarray(bf16_round(g), np.float32) * np.asarray(brq, np.float32)
    xp = bf16_round(np.asarray(xq, np.float32) + t)
    x64 = xp.astype(np.float64)
    mu = x64.mean(1, keepdims=True)
    var = (x64 * x64).mean(1, keepdims=True) - mu * mu
    return xp, (x64 - mu) / np.sqrt(var + 1e-6) * bf16_round(sc)


def rope_pairs(y, cos, sin):
    """Complex RoPE on adjacent pairs (2i, 2i+1): run_glue.py:27-32."""
    a, b = y[:, 0::2], y[:, 1::2]
    out = np.empty_like(y)
    out[:, 0::2] = a * cos - b * sin
    out[:, 1::2] = a * sin + b * cos
    return out


def rms_rope(x, w, cos, sin):
    """RMSNorm over the head dim (eps 1e-6) times w, then RoPE: run_glue.py:35-37."""
    x = np.asarray(x, np.float32)
    return rope_pairs(x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w, cos, sin)


def attention_f64(q, k, v, row_limit=None, nkv=None):
    """Float64 softmax attention on one head: run_attn.py:203-209 (non-causal, keys beyond nkv dropped) and
    run_attn.py:123-126 (per-row key limit: row j sees keys <= lim[j]). q (NQ, D), k/v (NK, D)."""
    q, k, v = (np.asarray(a, np.float64) for a in (q, k, v))
    if nkv is not None:
        k, v = k[:nkv], v[:nkv]
    s = q @ k.T / np.sqrt(q.shape[1])
    if row_limit is not None:
        s = np.where(np.arange(k.shape[0])[None, :] <= np.asarray(row_limit)[:, None], s, -np.inf)
    w = np.exp(s - s.max(1, keepdims=True))
    return (w / w.sum(1, keepdims=True)) @ v


def max_rel(got, ref):
    """max |got - ref| / max |ref|: the error statistic of run_ln.py:74-79."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def corr(got, ref):
    return float(np.corrcoef(np.asarray(got, np.float64).ravel(), np.asarray(ref, np.float64).ravel())[0, 1])
