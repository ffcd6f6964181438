/*
 * redline_b200.h - C ABI of the B200 (sm_100a) bfp16 weight-GEMM hot path.
 *
 * Drop-in boundary for Cukrus-directive/redline-tiny's matrix-multiply path. The reference crosses its device boundary
 * in Python, at `NPU.run(op, artifact, [iron tensors])` (redline/forward.py:138-165) and `gemm()`
 * (redline/forward.py:194-197); its data formats are defined by redline/npu_layouts.py and
 * redline/pack_weights.py. Each entry point below names the reference interface it replaces.
 *
 * Conventions (all entry points):
 *  - Plain device pointers and sizes; the caller owns every buffer (the reference's kernels also write caller-
 *    allocated iron tensors in place). Nothing here allocates device memory.
 *  - Calls are stream-ordered and asynchronous on `stream` (0 = the legacy default stream). Buffers must stay alive
 *    until the stream reaches the call (forward.py:151-153 states the same rule for the NPU).
 *  - Return 0 (RL_OK) or a negative rl_status; rl_last_error() gives the message (thread-local). Kernels never trap:
 *    a device-side failure (a bounded wait that ran out, a skipped out-of-range access) sets a device error word that
 *    rl_device_status() reads and clears.
 *  - bfp16 ("bfp16ebs8"): blocks of 8 consecutive values, 9 bytes each = [E][m0..m7], value = m * 2^(E - 133).
 *  - bf16 buffers are passed as uint16_t bit patterns.
 */
#ifndef REDLINE_B200_H
#define REDLINE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* rl_stream_t; /* the same handle as cudaStream_t / CUstream */

typedef enum {
  RL_OK = 0,
  RL_ERR_ARGUMENT = -1,    /* bad shape, null pointer or unknown enum */
  RL_ERR_ALIGNMENT = -2,   /* a pointer or a size breaks the documented alignment */
  RL_ERR_UNSUPPORTED = -3, /* valid request this build does not implement (e.g. no sm_100 device) */
  RL_ERR_CUDA = -4,        /* a CUDA runtime / driver call failed */
  RL_ERR_DEVICE = -5       /* rl_device_status: a kernel reported a device-side error */
} rl_status;

typedef enum { RL_F32 = 0, RL_BF16 = 1 } rl_dtype;

/* Stream order of 8-value blocks of an (M, K) matrix. RL_ROWMAJOR: block (r, c/8) at index r*K/8 + c/8.
 * RL_A_LAYOUT: the reference's GEMM A-operand order, a_layout(A, 128, 64) (npu_layouts.py:18-23; M % 128, K % 64).
 * RL_C_ATB: the order its GEMMs emit C and keep the residual stream in, c_layout_atb(C, 128, 128)
 * (npu_layouts.py:31-48; M % 512, K % 1024). */
typedef enum { RL_ROWMAJOR = 0, RL_A_LAYOUT = 1, RL_C_ATB = 2 } rl_layout;

typedef enum {
  RL_EPI_NONE = 0,   /* C = A @ B */
  RL_EPI_BIAS = 1,   /* C = A @ B + bias[N] */
  RL_EPI_SWIGLU = 2  /* weights packed with swiglu_interleaved=1; C[M, N/2] = silu(gate) * proj (+ bias first) */
} rl_epilogue;

/* Message of the last failed call on this host thread ("" if none). */
const char* rl_last_error(void);

/* Library version (major * 10000 + minor * 100 + patch). */
int rl_version(void);

/* Synchronise the current device, then read and clear the device error word (bit 1: a bounded wait ran out;
 * bit 2: a kernel-side range check skipped an access). Returns RL_ERR_DEVICE when any bit was set. */
int rl_device_status(int* flags_out);

/*
 * a1/a3 - activation quantiser. Replaces npu_layouts.to_bfp16 (redline/npu_layouts.py:62-88) applied to
 * a_layout(x, 128, 64) (npu_layouts.py:18-23), as forward.py:406 and forward.py:613 call it.
 * x: (M, K) row-major, dtype RL_F32 or RL_BF16, K % 8 == 0, 16-byte aligned.
 * q_out (may be NULL): M*K/8*9 bytes of bfp16, bit-identical to the reference, in `layout` order
 *   (RL_A_LAYOUT needs M % 128 == 0 and K % 64 == 0).
 * dq_out (may be NULL): the decoded values as bf16 (M, K) row-major - the A operand rl_linear_bfp16 takes.
 */
int rl_quantize_bfp16(const void* x, int x_dtype, int64_t M, int64_t K, int layout, uint8_t* q_out,
                      uint16_t* dq_out, rl_stream_t stream);

/*
 * a2 - decoder. Replaces npu_layouts.from_bfp16 (redline/npu_layouts.py:90-94) followed by a_unlayout
 * (npu_layouts.py:56-60) when layout == RL_A_LAYOUT. out: (M, K) row-major, RL_F32 or RL_BF16 (both exact).
 */
int rl_dequantize_bfp16(const uint8_t* q, int layout, int64_t M, int64_t K, void* out, int out_dtype,
                        rl_stream_t stream);

/*
 * a3/a5 - bf16 (M, K) between stream orders (row-major, a_layout, the ATB C order): the reference keeps its bf16
 * residual stream in the C order (run_ln.ln_pack_x, redline/run_ln.py:28-30; c_unlayout_atb for reading it back).
 */
int rl_permute_bf16(const uint16_t* src, int src_layout, uint16_t* dst, int dst_layout, int64_t M, int64_t K,
                    rl_stream_t stream);

/*
 * a4/a6 - the reference's packed-weight stream on the GPU. Replaces pack_weights.pack_b
 * (redline/pack_weights.py:72-79): out = to_bfp16(b_layout(B, 64, 128)), bit-identical.
 * B: (K, N) row-major (B = W^T, C = A @ B), RL_F32 or RL_BF16; K % 64 == 0, N % 128 == 0.
 */
int rl_pack_b(const void* B, int dtype, int64_t K, int64_t N, uint8_t* out, rl_stream_t stream);

/*
 * a6 - load-time repack of the reference's packed stream (the bytes of bNN_*.bin, pack_weights.py:106-112) into the
 * GPU-native tile format the GEMM streams. Lossless (the same blocks, reordered), 1.125 B per weight.
 * Native tile (128 columns x 64 K, 9216 B; N-tile outer, K-tile inner, like b_layout):
 *   bytes [0, 8192): mantissas in offset binary (m + 128), 16-byte chunk (j, n) at (j * 128 + n) * 16 = blocks 2j
 *                    and 2j+1 of column n;
 *   bytes [8192, 9216): exponents, column n at 8192 + n * 8, one byte per 8-row block.
 * swiglu_interleaved = 1: B is an up matrix with [gate 64 | proj 64] per 128-column tile (pack_weights.py:82-89);
 *   the native rows are permuted so each 32-row quarter holds 16 gate units then the same 16 proj units.
 */
int rl_weights_from_pack_b(const uint8_t* packed, int64_t K, int64_t N, int swiglu_interleaved, uint8_t* native,
                           rl_stream_t stream);

/* Pack float B (K, N) directly into the native format (equals rl_weights_from_pack_b(rl_pack_b(B))). */
int rl_pack_weights(const void* B, int dtype, int64_t K, int64_t N, int swiglu_interleaved, uint8_t* native,
                    rl_stream_t stream);

/*
 * Column shard `rank` of `world` of a packed B (K, N) for the N-split standalone GEMM: columns
 * [n0, n0 + n_cols) = [rank * N / world, (rank + 1) * N / world) are the contiguous bytes
 * [byte_offset, byte_offset + byte_count) of both the reference's pack_b stream and the native format, because both
 * store 128-column strips whole, N-tile outer (b_layout, redline/npu_layouts.py:11-16; pack_b,
 * redline/pack_weights.py:72-79). So a rank streams its shard in place, without repacking, and its GEMM output is
 * C[:, n0 : n0 + n_cols]. Needs K % 64 == 0 and N % (128 * world) == 0 (the 2-SM pair GEMM kernel also wants
 * n_cols % 256 == 0; other shards run the 1-SM kernel). Host arithmetic only: no device is touched. Up matrices
 * packed with swiglu_interleaved keep each [gate 64 | proj 64] tile whole, so a shard holds n_cols / 2 FFN units.
 */
int rl_weights_shard(int64_t K, int64_t N, int rank, int world, int64_t* n0, int64_t* n_cols, int64_t* byte_offset,
                     int64_t* byte_count);

/*
 * a7/a8/a9 - the packed-weight GEMM. Replaces gemm(npu, w, op, M, a, c) (redline/forward.py:194-197), which runs
 * matmul_vectorized_bfp16 (kernels/atb3/mm_bfp_rho.cc:64-177) and, for the up projection,
 * matmul_swiglu_bfp16 (kernels/atb3/mm_bfp_swiglu.cc:88-168).
 * x: (M, K) bf16 row-major holding bfp16-exact values (rl_quantize_bfp16's dq_out), 16-byte aligned, K % 64 == 0.
 * w_native: rl_weights_from_pack_b / rl_pack_weights output for B (K, N), N % 128 == 0.
 * bias: bf16 [N] or NULL (required for RL_EPI_BIAS).
 * out: (M, N) row-major (RL_EPI_SWIGLU: (M, N/2)), RL_BF16 or RL_F32. fp32 accumulation on tcgen05 tensor cores.
 */
int rl_linear_bfp16(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                    const uint16_t* bias, int epilogue, void* out, int out_dtype, rl_stream_t stream);

/* rl_linear_bfp16 with a caller workspace for split-K: when the pair kernel's grid would fill less than the GPU
 * (N % 256 == 0, few tiles, long K), K is split into S ranges whose fp32 partials go to the workspace and one
 * HBM-bound kernel adds them (+ bias) into out. rl_linear_bfp16_workspace(M, K, N, epilogue) gives the bytes
 * (S * M * N * 4; 0 when no split helps, or for the SwiGLU epilogue); with a smaller workspace, a NULL one or a
 * non-default kernel variant the call is rl_linear_bfp16. The result differs from the unsplit one only by fp32
 * summation order. */
size_t rl_linear_bfp16_workspace(int64_t M, int64_t K, int64_t N, int epilogue);
int rl_linear_bfp16_ws(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                       const uint16_t* bias, int epilogue, void* out, int out_dtype, void* workspace,
                       size_t workspace_bytes, rl_stream_t stream);

/*
 * a9/a13 - the SwiGLU MLP: quantise x (unless x_quantized), H = silu(x @ Bgate) * (x @ Bproj) rounded to bfp16
 * (the up GEMM with the SwiGLU epilogue), out = H @ Bdown. Replaces the up+SwiGLU / down pair of LM._layer
 * (redline/vlm_run.py:442-449) and CachedStep.blocks (redline/forward.py:250-251): matmul_swiglu_bfp16
 * (kernels/atb3/mm_bfp_swiglu.cc:88-168) followed by matmul_vectorized_bfp16.
 * x: (M, K) RL_BF16 / RL_F32 (x_quantized=1: bf16 already holding bfp16 values); w_up: native (K, F2) packed with
 * swiglu_interleaved=1, F2 = 2F; w_down: native (F, N); out: (M, N) RL_BF16 or RL_F32.
 * workspace: caller-owned device scratch of rl_swiglu_mlp_workspace(M, K, F, x_quantized) bytes, 256-byte aligned
 * (it includes room for the down GEMM's split-K partials when N = K; a workspace without it runs the down GEMM unsplit).
 */
size_t rl_swiglu_mlp_workspace(int64_t M, int64_t K, int64_t F, int x_quantized);
int rl_swiglu_mlp(const void* x, int x_dtype, int x_quantized, int64_t M, int64_t K, const uint8_t* w_up, int64_t F2,
                  const uint8_t* w_down, int64_t N, void* out, int out_dtype, void* workspace,
                  size_t workspace_bytes, rl_stream_t stream);

/*
 * No counterpart in the reference: rl_swiglu_mlp without a caller workspace, for callers that cannot allocate
 * device memory - a serving process that reserves its whole memory pool at start-up and treats any later
 * allocation as a failure, or a latency-critical path where cudaMalloc / cudaFree would synchronise the device.
 * Its scratch is a fixed 32 MiB device array inside this library (rl_swiglu_mlp_noalloc_capacity()), which every
 * GPU that loads the library holds until the process exits. The array must hold the quantised x (M x K bf16,
 * unless x_quantized) and H (M x F bf16), each rounded up to 256 bytes; requests whose two exceed 32 MiB return
 * RL_ERR_ARGUMENT. The down GEMM's split-K partials are used only when they fit in the rest of the array too
 * (otherwise it runs unsplit, with the same results up to fp32 summation order). The call allocates nothing.
 * The first call on each device looks up the array's device address (once, with that device current), so make
 * that first call before any stream capture; a cudaDeviceReset while the library is loaded invalidates that address
 * and is not supported. All calls share the one array: calls that overlap on the GPU (e.g. on two streams) race on
 * it. Nothing in it needs to start zeroed - each call writes everything it reads. Arguments as rl_swiglu_mlp.
 */
size_t rl_swiglu_mlp_noalloc_capacity(void);
int rl_swiglu_mlp_noalloc(const void* x, int x_dtype, int x_quantized, int64_t M, int64_t K, const uint8_t* w_up,
                          int64_t F2, const uint8_t* w_down, int64_t N, void* out, int out_dtype,
                          rl_stream_t stream);

/*
 * a10 - residual + gate + LayerNorm + modulate between the GEMMs. Replaces the ln_mod artifact
 * (kernels/glue/ln_mod.cc:92-204, run by forward.py:249, 253, 259) and its numpy model redline/run_ln.py:65-71:
 *   x' = bf16(x + g * branch)            (float32 arithmetic, one bf16 rounding; bit-exact with run_ln.ln_ref)
 *   y  = (x' - mean) / sqrt(var + 1e-6) * sc, rounded to bfp16 blocks of 8 along the row.
 * x: (M, D) bf16 row-major; branch (NULL = zero branch): (M, D) row-major, RL_BF16, or RL_F32 (e.g. the sum of
 * tensor-parallel partial GEMM outputs; rounded to bf16 on load); params: bf16 (2, 2, D) = two rows [g | sc], the layout of
 * run_ln.ln_params (run_ln.py:38-40); rows r < row_split use parameter row 1 (the reference's S * 128 split).
 * Outputs (each may be NULL): x_out (M, D) bf16 = x'; y_dq (M, D) bf16 = decoded y (the next GEMM's A operand);
 * y_q = y's bfp16 bytes, row-major blocks.
 */
int rl_ln_mod(const uint16_t* x, const void* branch, int branch_dtype, const uint16_t* params, int64_t M, int64_t D,
              int64_t row_split, uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream);

/*
 * RMSNorm residual glue of the Qwen3-VL text encoder. Replaces the vlm-rms / vlm-rms16 artifacts
 * (kernels/vlm/rms_mod.cc, run by redline/vlm_run.py:340-341) and is checked against vlm_run.rms_ref
 * (vlm_run.py:68-71): x' = bf16(x + g * branch), y = x' / sqrt(mean(x'^2) + 1e-6) * sc, rounded to bfp16 blocks of
 * 8. Arguments, parameter rows and outputs as rl_ln_mod (the reference's rms_params have g = 1).
 */
int rl_rms_mod(const uint16_t* x, const void* branch, int branch_dtype, const uint16_t* params, int64_t M, int64_t D,
               int64_t row_split, uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream);

/*
 * a11 - QK-RMSNorm + RoPE. Replaces the qkv_post artifact (kernels/glue/qkv_post.cc:112-178, run by forward.py:246)
 * and run_glue.rms_rope (redline/run_glue.py:27-37): per token and head, q and k are RMS-normalised over their 128
 * dims (eps 1e-6), scaled by w_q / w_k, and rotated on adjacent pairs (2i, 2i+1) by the token's (cos, sin).
 * qkv: (M, 3 * H * 128) bf16 = [q heads | k heads | v heads] (the QKV GEMM output); rope_cs: float32 (M, 64, 2),
 * the table of host_glue.rope (redline/host_glue.py:68-91); w_q, w_k: float32 [128].
 * Out: q, k (H, M, 128) bf16; vt (H, 128, ldv) bf16 = V transposed (keys contiguous), columns M..ldv-1 zeroed;
 * ldv >= M, ldv % 8 == 0.
 */
int rl_qkv_post(const uint16_t* qkv, const float* rope_cs, const float* w_q, const float* w_k, int64_t M, int H,
                uint16_t* q, uint16_t* k, uint16_t* vt, int64_t ldv, rl_stream_t stream);

/*
 * rl_qkv_post for grouped-query attention: qkv (M, (H + 2 Hkv) * 128) = [q H heads | k Hkv heads | v Hkv heads]
 * (the Qwen3-VL layer, redline/vlm_run.py:407-412, kernels/vlm/qkv_gqa_design.py). Out: q (H, M, 128), k (Hkv, M,
 * 128), vt (Hkv, 128, ldv). rl_qkv_post(..., H, ...) is this with Hkv = H.
 */
int rl_qkv_post_gqa(const uint16_t* qkv, const float* rope_cs, const float* w_q, const float* w_k, int64_t M, int H,
                    int Hkv, uint16_t* q, uint16_t* k, uint16_t* vt, int64_t ldv, rl_stream_t stream);

/*
 * The QKV projection with rl_qkv_post_gqa in its epilogue: one GEMM launch in place of rl_linear_bfp16 + rl_qkv_post
 * (forward.py:245-246, the qkv_bfp artifact followed by kernels/glue/qkv_post.cc:112-178; redline/vlm_run.py:407-412
 * for grouped-query heads). x: (M, K) bf16; w_native: the packed (K, (H + 2 Hkv) * 128) QKV weight (K % 64 == 0;
 * an even head count runs on the 2-SM pair kernel, an odd one on the 1-SM kernel). The accumulator of each head is rounded to bf16 (the projection's output dtype) and then normalised,
 * rotated and stored as rl_qkv_post_gqa stores it: q (H, M, 128), k (Hkv, M, 128), vt (Hkv, 128, ldv) with columns
 * M..ldv-1 zeroed. ldv % 16 == 0 and M <= ldv <= M rounded up to a multiple of 256. Never splits K.
 */
int rl_qkv_linear(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int H, int Hkv,
                  const float* rope_cs, const float* w_q, const float* w_k, uint16_t* q, uint16_t* k, uint16_t* vt,
                  int64_t ldv, rl_stream_t stream);

/*
 * a12 - joint text+image flash attention, head_dim 128, on tcgen05. Replaces the attention artifacts
 * (kernels/attn/attn_bfp.cc:846-923, run by forward.py:247, 369, 603) and is checked against the float64 softmax of
 * redline/run_attn.py:203-209 (key-tail mask, run_attn.py:153-155) and run_attn.py:123-126 (per-row key limits).
 * q: (H, Nq, 128), k: (H, Nk, 128), vt: (H, 128, ldv) bf16 (rl_qkv_post's outputs); keys >= nkv are masked;
 * row_limit (may be NULL): int32 [Nq], query row r sees keys <= row_limit[r]; logits = (q . k) * scale_log2 in log2
 * units (log2(e)/sqrt(128) for unscaled q; 1.0 when q already carries it, as the reference's w_q does).
 * o: (Nq, ldo) bf16, head h at columns [128h, 128h + 128), rounded to bfp16 blocks of 8 (the out-projection's A
 * operand). Rows with no visible key are zero.
 */
int rl_attention(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int64_t Nq,
                 int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, uint16_t* o, int64_t ldo,
                 rl_stream_t stream);

/*
 * Grouped-query attention (the Qwen3-VL causal attention, kernels/vlm/attn_causal.cc, checked in the reference by
 * vlm_run.attn_ref, vlm_run.py:181-190): H query heads over Hkv K/V heads, query head h reads K/V head
 * h / (H / Hkv); k (Hkv, Nk, 128), vt (Hkv, 128, ldv); causal = row_limit[r] = r. rl_attention is this with Hkv = H.
 */
int rl_attention_gqa(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int Hkv,
                     int64_t Nq, int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, uint16_t* o,
                     int64_t ldo, rl_stream_t stream);

/* rl_attention_gqa with o (Nq, ldo) fp32 = O / l before its bfp16 rounding (ldo % 8 == 0, 16-byte aligned): the
 * attention kernel's own result, for callers that keep the output in fp32 and for checks of the kernel against the
 * float64 softmax without the output rounding in between (run_attn.py:203-209 compares the same quantity). */
int rl_attention_gqa_f32(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int Hkv,
                         int64_t Nq, int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, float* o,
                         int64_t ldo, rl_stream_t stream);

/*
 * VAE decoder convolution, 3x3 pad 1 (taps = 3) or 1x1 (taps = 1), stride 1, with bfp16 weights. Replaces the vconv
 * artifacts (kernels/vae/vconv.cc:1-17, redline/vae_decode.py:168-194; weights packed by vae_ops.pack_vconv,
 * vae_ops.py:44-61) and is checked against vae_ops.conv_ref (vae_ops.py:64-75).
 * x: (H, W, Cin) bf16 holding bfp16-exact values (rl_quantize_bfp16's decoded output of the (H * W, Cin) matrix);
 * Cin % 8 == 0. w_native: the native tiles of B = [(dy * taps + dx) * Kt + ci][co] = w[co][ci][dy][dx], Kt = Cin
 * rounded up to a multiple of 64 (zero rows for Cin <= ci < Kt), K = taps^2 * Kt; N = Cout, a multiple of 128 (pad
 * smaller outputs with zero columns); bias: bf16 [Cout] or NULL; out: (H, W, Cout) bf16. With W % 128 == 0 and
 * Cin >= 64 the GEMM loads its A tiles from x directly (implicit GEMM, TMA zero fill as the padding) and needs no
 * workspace; otherwise the rows are gathered first into the workspace: rl_conv2d_workspace(H, W, Cin, taps) bytes
 * (0 when nothing is gathered: the implicit GEMM, or a 1x1 conv with Cin % 64 == 0).
 * rl_set_conv_path(1) forces the gather for every shape (0: the default choice); it returns the previous setting.
 */
size_t rl_conv2d_workspace(int H, int W, int Cin, int taps);
int rl_set_conv_path(int path);
int rl_conv2d_bfp16(const uint16_t* x, int H, int W, int Cin, const uint8_t* w_native, int Cout, int taps,
                    const uint16_t* bias, uint16_t* out, void* workspace, size_t workspace_bytes,
                    rl_stream_t stream);

/* Per-step adaLN conditioning of the DiT (host_glue.py:31-48, forward.py:231-238), run on the GPU so the denoise
 * step needs no host matrix work:
 * rl_matvec_f32: y[r][n] = sum_k f(x[r][k]) w[n][k] (+ bias[n]) for r < R <= 4, f = SiLU when silu_in; w fp32
 *   row-major (N, K), K % 4 == 0, R * K <= 12288; the linear_1 / linear_2 / modulation / norm_out products.
 * rl_sinusoidal_embed: e (2, 2 * half) = [cos(t_r f_i) | sin(t_r f_i)] for rows t_0, t_1 (the timestep times 1000)
 *   and frequencies f (half).
 * rl_adaln_params: from mod (2, 4D) = [scale1 | gate1 | scale2 | gate2] and out_scale (2 rows of ld_out >= D; the
 *   first D columns are used), the bf16 LayerNorm
 *   parameter sets (2, 2, D) = rows [g | sc]: first (1, 1 + scale1), mlp (tanh gate1, 1 + scale2),
 *   attn (tanh gate2, 1 + scale1), out (tanh gate2, 1 + out_scale). */
int rl_matvec_f32(const float* w, int N, int K, const float* x, int R, const float* bias, int silu_in, float* y,
                  rl_stream_t stream);
int rl_sinusoidal_embed(float t0, float t1, const float* freqs, int half, float* e, rl_stream_t stream);
int rl_adaln_params(const float* mod, const float* out_scale, int ld_out, int D, uint16_t* first, uint16_t* mlp,
                    uint16_t* attn, uint16_t* out, rl_stream_t stream);

/* The reference's NPU attention formats, for the QKV-post and attention artifacts of its DiT (forward.py:209-412):
 * per head h and 64-token tile t, Q[h][t] = to_bfp16(a_layout(Q_h tile, 64, 128)) and KV[h][t] = [K | V] with
 * K = to_bfp16(b_layout(K_tile^T, 128, 64)), V = to_bfp16(b_layout(V_tile, 64, 128)) (run_attn.py:29-35, 82-92),
 * 9216 bytes per tile.
 * rl_npu_qkv_pack: from q, k (H, 64T, 128) and vt (H, 128, ldv) bf16 -> q_out (H, T, 9216 B), kv_out (H, T, 2, 9216 B).
 * rl_npu_q_unpack: Q tiles [tile0, tile0 + ntiles) of each head (tiles_per_head in the buffer) -> q (H, 64 ntiles, 128).
 * rl_npu_kv_unpack: K/V tiles [tile0, tile0 + ntiles) of each head -> keys key0 .. key0 + 64 ntiles of k (H, nk, 128)
 *   and vt (H, 128, ldv) (key0 % 8 == 0, nk <= ldv, ldv % 8 == 0).
 * rl_npu_qkv_tables: the QKV-post table (T, 8448) bf16 (run_qkv.qkv_tables, run_qkv.py:60-72) -> rope_cs (64T, 64, 2)
 *   float (cos, sin per row and rotary pair), w_q, w_k (128 floats each). */
int rl_npu_qkv_pack(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int T,
                    uint8_t* q_out, uint8_t* kv_out, rl_stream_t stream);
int rl_npu_q_unpack(const uint8_t* q_in, int H, int tiles_per_head, int tile0, int ntiles, uint16_t* q,
                    rl_stream_t stream);
int rl_npu_kv_unpack(const uint8_t* kv_in, int H, int tiles_per_head, int tile0, int ntiles, int64_t key0,
                     int64_t nk, int64_t ldv, uint16_t* k, uint16_t* vt, rl_stream_t stream);
int rl_npu_qkv_tables(const uint16_t* tables, int T, float* rope_cs, float* w_q, float* w_k, rl_stream_t stream);

/* Tensor-parallel residual + LayerNorm with the row-split projection's all-reduce fused in (the reference runs on one
 * device; the TP DiT adds the out- and down-projection partials across ranks once per sublayer). Every rank's projection writes its bf16 (M, D)
 * partial, in rl_linear_bfp16_partial's chunk layout, into a peer-readable buffer (rl_ipc_alloc); rl_tp_signal stores `epoch` into entry [slot][rank] of every rank's signal pad
 * (pads: device array of W pointers to the pads' bases, each W x nslots uint64, zero before first use);
 * rl_ln_mod_tp (rl_ln_mod's math with the branch = bf16 of the fp32 sum, in rank order, of the W partials `parts`, a
 * device array of W pointers) first waits until this rank's pad (`pad` = its base + slot * W) holds >= epoch for
 * every other rank - a bounded wait that records a device error when it runs out. Epochs increase by one per use of
 * a slot; two slots used alternately keep a rank's next write of a partial after every rank's read of it. */
/* Peer-readable device buffers for the fused reduction: rl_ipc_alloc returns a zeroed cudaMalloc allocation and its
 * 64-byte CUDA IPC handle; the other ranks map it with rl_ipc_open (rl_ipc_close unmaps it, rl_ipc_free frees the
 * owner's allocation). */
int rl_ipc_alloc(int64_t bytes, void** ptr, void* handle);
int rl_ipc_open(const void* handle, void** ptr);
int rl_ipc_close(void* ptr);
int rl_ipc_free(void* ptr);
/* rl_linear_bfp16 with bf16 output (no SwiGLU) that also stores every output value at the same offset of `mirror`
 * (a second M x N bf16 buffer, e.g. a peer GPU's mapping): the tensor-parallel projection sends its partial to the
 * other rank while the GEMM runs. */
int rl_linear_bfp16_mirror(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                           const uint16_t* bias, int epilogue, void* out, void* mirror, int out_dtype,
                           rl_stream_t stream);
/* The tensor-parallel projection's partial C = x @ B (bf16, no bias) in the partial layout rl_ln_mod_tp reads:
 * 16-row x 32-column chunks of 512 values (1 KB), chunk (r / 16, c / 32) at element ((r / 16) * N / 32 + c / 32) * 512,
 * element (r % 16) * 32 + c % 32 inside it. out, and mirror when not NULL (the other rank's buffer), hold
 * ceil(M / 16) * 16 rows; each chunk goes to the mirror as one 1 KB bulk copy while the GEMM runs (sixteen times
 * fewer, larger NVLink writes than rl_linear_bfp16_mirror's row segments). */
int rl_linear_bfp16_partial(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                            uint16_t* out, uint16_t* mirror, rl_stream_t stream);
int rl_tp_signal(void* const* pads, int W, int rank, int slot, unsigned long long epoch, rl_stream_t stream);
/* Tensor-parallel reduce-scatter + row-sharded LayerNorm + all-gather over peer memory (W ranks, each owning R = M / W
 * consecutive rows; R % 16 == 0). rl_linear_bfp16_scatter: the projection's bf16 partial in rl_linear_bfp16_partial's
 * chunk layout, restarted at row o R for each owner o and stored as whole 1 KB bulk copies to dsts[o] (a device array
 * of W pointers: rank o's receive buffer for this rank's partial; peers over NVLink); every value crosses to its
 * owner once. rl_ln_mod_tp_rs: rl_ln_mod_tp over this rank's R rows (x, x_out: R x D; parts: the W received partials,
 * R-row chunk layout, summed in rank order; row_split relative to the block) that stores y into every rank's copy of
 * the next GEMM's A operand (y_dsts: device array of W pointers to row r0 = rank x R of each copy). Every pointer
 * inside dsts, parts and y_dsts must be 16-byte aligned (the kernels cannot check device-resident pointers; a
 * cudaMalloc / rl_ipc_alloc base plus offsets that are multiples of 16 bytes, as tp.PeerRS builds them). rl_tp_wait: a
 * bounded wait on the stream until every other rank's entry of pad (this rank's, W uint64) reaches epoch; it runs
 * between rl_tp_signal of the all-gather and the GEMM that reads the gathered rows. On a timeout the kernel records
 * the error for rl_device_status and returns. */
int rl_linear_bfp16_scatter(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                            uint16_t* const* dsts, int W, int64_t rows_per_rank, rl_stream_t stream);
int rl_ln_mod_tp_rs(const uint16_t* x, const uint16_t* const* parts, int W, const unsigned long long* pad, int rank,
                    unsigned long long epoch, const uint16_t* params, int64_t R, int64_t D, int64_t row_split,
                    uint16_t* x_out, uint16_t* const* y_dsts, rl_stream_t stream);
int rl_tp_wait(const unsigned long long* pad, int W, int rank, unsigned long long epoch, rl_stream_t stream);
int rl_ln_mod_tp(const uint16_t* x, const uint16_t* const* parts, int W, const unsigned long long* pad, int rank,
                 unsigned long long epoch, const uint16_t* params, int64_t M, int64_t D, int64_t row_split,
                 uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream);

/* GEMM kernel variant for tests and benchmarks: 0 = default (the 2-SM pair kernel with weights decoded into TMEM
 * when N is a multiple of 256, else variant 2), 1 = 1-SM, weights decoded into shared memory (MMA A operand from
 * shared memory), 2 = 1-SM, weights decoded into tensor memory (A from TMEM), 3 / 4 = 2-SM pair kernel
 * (tcgen05.mma cta_group::2 over a cluster of two CTAs) with A in shared memory / TMEM; tuning codes
 * 1000*P + 100*G + 10*V + S (1313, 1125, 2125, 1224, 2224, 1333, 1234, 1346, 1448, 2248) also select the decode split
 * and the pipeline depth. Returns the previous value. */
/* Resident 2-CTA clusters of the default pair GEMM kernel on the current device (two CTAs of a cluster share a GPC,
 * so this follows the chip's GPC layout); 0 without an sm_100 device. The split-K choice uses it. */
int rl_gemm_pair_clusters(void);
int rl_set_gemm_variant(int variant);

/* Attention kernel for tests and benchmarks: 0 = default (two 128-query tiles per CTA, the tensor pipe working on one
 * tile while the other's softmax runs; = variant 5), 1 = one query tile per CTA, 2-5 = two-tile forms (2 + 2 * the
 * next Q.K issued in order behind the P.V instead of after its completion + P released in two halves). Returns the
 * previous value. */
int rl_set_attention_variant(int variant);

#ifdef __cplusplus
}
#endif

#endif /* REDLINE_B200_H */
