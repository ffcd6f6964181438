// Packed-weight bfp16 GEMM on tcgen05 tensor cores (sm_100a).
//
// Computes C[M, N] = X[M, K] @ B[K, N] where X is bf16 holding bfp16-exact values and B is streamed in the native
// packed tile format (1.125 B per weight; see rl_weights_from_pack_b). The weights sit on the MMA's M side:
//   D^T tile [128 weight columns (TMEM lanes)] x [256 activation rows (TMEM columns)], fp32 in tensor memory,
//   D^T += W^T[128 x K] * X[256 x K]^T, issued as tcgen05.mma kind::f16 M=128 N=256 K=16.
// Per 64-deep K step a pipeline stage holds
//   X tile   256 x 64 bf16, loaded by TMA with the 128-byte swizzle (the MMA's B operand, K-major);
//   W9 tile  128 x 64 bfp16 in native order, 9216 contiguous bytes, loaded by one bulk copy;
// and expander warps decode the W9 tile to bf16 (exact: int8 * 2^e fits bf16) into the MMA's A operand:
//   variant kSmemA: a 128 x 64 bf16 tile in shared memory, in the 128-byte-swizzled K-major layout;
//   variant kTmemA: tensor memory, one lane per weight column, 2 bf16 per 32-bit column (tcgen05.st), which keeps
//                   the decoded operand out of shared memory entirely (no write, no MMA re-read).
// Decoding is the throughput limiter (16 weights per MMA cycle per SM), so it is spread over 4*P*G warps: P parts
// split one stage's eight 8-deep blocks, G groups take alternate stages.
// Warp roles: warp 0 = TMA producer + TMEM allocator, warp 1 = MMA issuer (warp-wide loop, elected lane issues),
// then the expanders, then 8 epilogue warps (tcgen05.ld of D, bias / SwiGLU, transposed through shared memory into
// row-major C). The accumulator is single-buffered in TMEM (the decoded A stages take the rest), so two warps per
// lane quarter drain it in halves and release it as soon as their last tcgen05.ld has landed, before the last stores.
// The kernel is persistent: one CTA per SM walks tiles (activation-tile fastest, so the CTAs in flight share the
// same weight columns and the whole X in L2).
#include <cmath>
#include <mutex>

#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace gemm {

constexpr int BM = 128;                 // weight columns per tile = MMA M = TMEM lanes
constexpr int BN = 256;                 // activation rows per tile = MMA N
constexpr int BK = 64;                  // K per pipeline stage
constexpr int UK = 16;                  // K per tcgen05.mma (kind::f16)
constexpr int X_BYTES = BN * BK * 2;    // 32768
constexpr int WE_BYTES = BM * BK * 2;   // 16384 (decoded weights, shared-memory variant)
constexpr int W9_BYTES = 9216;          // one native weight tile
constexpr int kChunk = 16;              // epilogue: D columns (activation rows) per tcgen05.ld
constexpr int kSwStride = 36;           // SwiGLU staging row stride (floats): 16-byte rows without bank conflicts
constexpr int kEpiStageBytes = kChunk * kSwStride * 4;  // per epilogue warp: 16 rows x 32 columns x fp32 (+pad)

enum Variant { kSmemA = 1, kTmemA = 2 };

template <int V, int S, int G, int P>
struct Cfg {
  static constexpr int kStages = S;
  static constexpr int kGroups = G;
  static constexpr int kParts = P;
  static constexpr int kExpWarps = 4 * P * G;
  static constexpr int kEpiWarps = 8;                                          // 2 per TMEM lane quarter
  static constexpr int kWarps = 2 + kExpWarps + kEpiWarps;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kEpiWarp0 = 2 + kExpWarps;
  static constexpr int kXOff = 0;                                              // S x 32 KB, 1024-aligned
  static constexpr int kWEOff = kXOff + S * X_BYTES;                           // SS: S x 16 KB, 1024-aligned
  static constexpr int kW9Off = kWEOff + (V == kSmemA ? S * WE_BYTES : 0);     // S x 9216 B, 16-aligned
  static constexpr int kEpiOff = kW9Off + S * W9_BYTES;
  static constexpr int kBarOff = kEpiOff + kEpiWarps * kEpiStageBytes;
  static constexpr int kAccBufs = (V == kSmemA) ? 2 : 1;                       // TMEM D buffers of 256 columns
  static constexpr int kTmemACol = 256;                                        // TS: A stages after one D buffer
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kBarOff + 256;
  static_assert(V == kSmemA || 256 + S * (BK / 2) <= 512, "TMEM: one D buffer + S A stages");
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(S <= 8 && G >= 1 && G <= 4 && (P == 1 || P == 2), "config");
  // A decoder group takes the stages s with s % G == its group, so that it waits on every phase of those stages'
  // load barriers in turn. With S % G != 0 a group would return to a stage only every lcm(S, G) K steps, and its
  // parity wait could be satisfied by a phase two behind the one it needs when a later load lands first.
  static_assert(S % G == 0, "the decoder groups must own whole stages");
};

struct Params {
  const uint8_t* w9;     // native weight tiles
  const uint16_t* bias;  // bf16 [N] or null
  void* out;
  int64_t M, N, K;
  int out_f32;           // 1: fp32 output, 0: bf16
  int epilogue;          // RL_EPI_*
  int num_x_tiles, num_w_tiles, num_tiles, KT;
  int splits;            // pair kernel: K split into this many ranges, fp32 partials split_stride elements apart
  int64_t split_stride;
  int group_x = 0;       // pair kernel tile order: groups of group_x activation tiles (0: one group; pair_tile_coords)
  void* mirror = nullptr;  // bf16 output without SwiGLU: every 16-byte store of `out` is repeated here (same layout;
                           // a peer GPU's buffer for the tensor-parallel reduction)
  int chunked = 0;         // bf16 output in 16-row x 32-column chunks of 1 KB (the tensor-parallel partial layout)
  // chunked output scattered by rows (the tensor-parallel reduce-scatter): rows [o R, o R + R) go, as whole 1 KB
  // chunks in the same layout restarted at row o R, to scatter[o] (rank o's receive buffer; peers over NVLink)
  uint16_t* const* scatter = nullptr;
  int64_t scatter_rows = 0;
  // QKV projection with QK-RMSNorm + RoPE in the epilogue (qkv_H > 0): the weight tiles are [q heads | k heads |
  // v heads] of 128 columns each; q / k tiles are RMS-normalised per token over their 128 columns (eps 1e-6), scaled
  // by w_q / w_k and rotated on adjacent column pairs by rope_cs (M, 64, 2) = (cos, sin), written to q_out / k_out
  // (heads, M, 128); v tiles are written transposed to vt_out (Hkv, 128, ldv), tokens contiguous.
  int qkv_H = 0, qkv_Hkv = 0;
  const float* rope_cs = nullptr;
  const float* w_q = nullptr;
  const float* w_k = nullptr;
  uint16_t* q_out = nullptr;
  uint16_t* k_out = nullptr;
  uint16_t* vt_out = nullptr;
  int64_t ldv = 0;
  // Convolution (implicit GEMM) when conv_W > 0: the A rows are the pixels of an (H, W, C) image (W % 128 == 0), the
  // tensor map is 3-D over (C, W, H), and K step kt covers channels 64 (kt % conv_cpt) .. + 63 of tap kt / conv_cpt
  // (taps in (dy, dx) row-major order, conv_cpt = ceil(C / 64) steps per tap).
  int conv_W = 0, conv_H = 0, conv_C = 0, conv_taps = 0, conv_cpt = 0;
};

// Conv mode: the 128 A rows starting at pixel pix0 (one image row, since W % 128 == 0) for K step kt, read from the
// image at the tap's offset; TMA's zero fill outside the (C, W, H) box is the convolution's zero padding (the
// innermost coordinate is a multiple of 64 channels and never negative; the others may be -1 or W / H).
__device__ __forceinline__ void load_conv_rows(void* dst, const CUtensorMap* map, uint64_t* bar, const Params& p,
                                               int kt, int pix0) {
  const int tap = kt / p.conv_cpt, cb = kt - tap * p.conv_cpt;
  const int half = p.conv_taps >> 1;
  const int dy = tap / p.conv_taps - half, dx = tap % p.conv_taps - half;
  const int h = pix0 / p.conv_W, w = pix0 - h * p.conv_W;
  tma_load_3d(dst, map, bar, cb * BK, w + dx, h + dy);
}

struct Barriers {
  uint64_t full[8];      // producer tx: X + W9 landed
  uint64_t expf[8];      // expanders: decoded A stage ready
  uint64_t empty[8];     // MMA commit: stage consumed
  uint64_t accf[2];      // MMA commit: accumulator complete
  uint64_t acce[2];      // epilogue: accumulator drained
  uint64_t drain;        // error path: wait for MMAs in flight
  uint64_t rms[2];       // QKV epilogue: the 4 epilogue warps of column half h have posted their sums of squares
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

// silu with the fast intrinsics (error ~1e-6 relative, far below the bfp16 step the result is rounded to)
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Epilogue of one 16-column chunk of D (16 activation rows x this warp's 32 weight columns): bias, SwiGLU or plain
// conversion, transposed through the warp's staging buffer into row-major global memory.
__device__ __forceinline__ void epilogue_chunk(const Params& p, const uint32_t (&r)[kChunk], uint8_t* st, int lane,
                                               int q, int wt, int64_t x0, float bias_v, int64_t out_off = 0) {
  if (p.epilogue == RL_EPI_SWIGLU) {
    // lanes 0-15 hold the gate of units 16q + lane, lanes 16-31 the proj of the same units. Stage the chunk
    // (16 rows x 32 values, row stride 36 floats: conflict-free both ways), then lane (row = lane & 15,
    // half = lane >> 4) owns 8 consecutive units of one row - one bfp16 block, so the block maximum is local.
    float* s32 = reinterpret_cast<float*>(st);
#pragma unroll
    for (int j = 0; j < kChunk; ++j) s32[j * kSwStride + lane] = __uint_as_float(r[j]) + bias_v;
    __syncwarp();
    const int rr = lane & 15, part = lane >> 4;
    const float4* rowp = reinterpret_cast<const float4*>(s32 + rr * kSwStride + 8 * part);
    const float4 g0 = rowp[0], g1 = rowp[1], p0 = rowp[4], p1 = rowp[5];   // proj is 16 floats to the right
    const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    uint32_t hb[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) hb[i] = __float_as_uint(silu_f(gv[i]) * pv[i]);
    uint32_t E, lo, hi, w[4];
    bfp16_quant_block_fast(hb, E, lo, hi, w);
    const int64_t Nout = p.N / 2;
    const int64_t xr = x0 + rr;
    if (xr < p.M)
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + xr * Nout + static_cast<int64_t>(wt) * 64 + 16 * q +
                                8 * part) = make_uint4(w[0], w[1], w[2], w[3]);
    __syncwarp();
  } else if (!p.out_f32) {
    uint16_t* s16 = reinterpret_cast<uint16_t*>(st);
#pragma unroll
    for (int j = 0; j < kChunk; j += 2) {
      uint32_t pr;   // rows j (low half) and j + 1 (high half), rounded to nearest even in one instruction
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pr) : "f"(__uint_as_float(r[j + 1]) + bias_v),
          "f"(__uint_as_float(r[j]) + bias_v));
      s16[j * 32 + lane] = static_cast<uint16_t>(pr);
      s16[(j + 1) * 32 + lane] = static_cast<uint16_t>(pr >> 16);
    }
    __syncwarp();
    uint16_t* outp = static_cast<uint16_t*>(p.out);
    if (p.chunked) {
      // the tensor-parallel partial layout: the staged 16 x 32 chunk is one contiguous KB, chunk (x0 / 16,
      // column / 32) - written whole here (the buffers hold the last chunk row's padding rows too; chunks wholly
      // past M are skipped) and, to the mirror, as one 1 KB bulk copy instead of sixteen 64-byte rows
      if (p.scatter) {
        if (x0 < p.M) {
          const int64_t o = x0 / p.scatter_rows;
          const int64_t chunk = ((x0 - o * p.scatter_rows) >> 4) * (p.N >> 5) +
                                ((static_cast<int64_t>(wt) * BM + 32 * q) >> 5);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            bulk_store(p.scatter[o] + chunk * 512, s16, 1024);
            bulk_commit();
            bulk_store_wait_read();
          }
        }
        __syncwarp();
        return;
      }
      if (x0 < p.M) {
        const int64_t chunk = (x0 >> 4) * (p.N >> 5) + ((static_cast<int64_t>(wt) * BM + 32 * q) >> 5);
        uint4* dst = reinterpret_cast<uint4*>(outp + chunk * 512);
        dst[lane] = reinterpret_cast<const uint4*>(s16)[lane];
        dst[lane + 32] = reinterpret_cast<const uint4*>(s16)[lane + 32];
        if (p.mirror) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            bulk_store(static_cast<uint16_t*>(p.mirror) + chunk * 512, s16, 1024);
            bulk_commit();
            bulk_store_wait_read();
          }
        }
      }
      __syncwarp();
      return;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = lane + 32 * i, rr = idx >> 2, part = idx & 3;
      const int64_t xr = x0 + rr;
      if (xr < p.M)
        *reinterpret_cast<uint4*>(outp + xr * p.N + static_cast<int64_t>(wt) * BM + 32 * q + part * 8) =
            reinterpret_cast<const uint4*>(s16 + rr * 32)[part];
    }
    if (p.mirror) {
      // the staged chunk again into the mirror (a peer GPU's buffer): one 64-byte bulk copy per row, so the
      // copy engine of the SM carries the NVLink stores and the warp waits only until the chunk has been read
      // (addresses: staging rows 64 bytes apart in a 16-byte aligned buffer; global rows start at column
      // wt * 128 + 32 q of a row of N % 128 == 0 bf16 values - all 64-byte aligned)
      fence_proxy_async_smem();
      __syncwarp();
      if (lane < 16) {
        const int64_t xr = x0 + lane;
        if (xr < p.M) {
          bulk_store(static_cast<uint16_t*>(p.mirror) + xr * p.N + static_cast<int64_t>(wt) * BM + 32 * q,
                     s16 + lane * 32, 64);
          bulk_commit();
          bulk_store_wait_read();
        }
      }
    }
    __syncwarp();
  } else {
    float* s32 = reinterpret_cast<float*>(st);
    float* outp = static_cast<float*>(p.out) + out_off;
#pragma unroll
    for (int j = 0; j < kChunk; ++j) s32[j * 32 + lane] = __uint_as_float(r[j]) + bias_v;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = lane + 32 * i, rr = idx >> 3, part = idx & 7;
      const int64_t xr = x0 + rr;
      if (xr < p.M)
        *reinterpret_cast<uint4*>(outp + xr * p.N + static_cast<int64_t>(wt) * BM + 32 * q + part * 4) =
            reinterpret_cast<const uint4*>(s32 + rr * 32)[part];
    }
    __syncwarp();
  }
}

// ---- QKV epilogue: QK-RMSNorm + RoPE on the accumulator (restates kernels/glue/qkv_post.cc:112-178 and
// redline/run_glue.py:27-37 as the separate rl_qkv_post does: inv = 1 / sqrt(sum of squares / 128 + 1e-6), n = x * inv
// * w, (n0 cos - n1 sin, n0 sin + n1 cos) on columns (2i, 2i + 1)). A 128-column weight tile is one head; the four
// epilogue warps of a column half each hold 32 of its columns for the same tokens, so they post their per-token
// sums of squares in their staging buffers and meet on an mbarrier (bounded wait) before any of them normalises.
// The epilogue staging buffer of a warp: [0, 1024) the bf16 tile of a pass-1 chunk, then 1 / rms of the half's 128
// tokens in pass 2; [1024, 2048) this warp's 128 per-token sums of squares, two buffers by tile parity (another warp
// of the half may still read tile t's sums while this one posts tile t + 1's: the accumulator it needs for t + 1 is
// released only after every warp's pass 1, and tile t + 2 needs every warp's pass 1 of t + 1, after its read of t).
constexpr int kQkvRstdOff = 0;
constexpr int kQkvPartOff = 1024;
static_assert(kQkvPartOff + 2 * 512 <= kEpiStageBytes, "QKV epilogue staging");
constexpr int kQkvU = 2;            // pass 2: tokens per lane whose loads are in flight together

// The warp-wide sum of v[j] for each of 16 tokens j (a transposing butterfly, 16 shuffles): lanes 2t and 2t + 1
// return the sum for token t.
__device__ __forceinline__ float warp_sum16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 8], keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 4], keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    const float send = up ? v[i] : v[i + 2], keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// The epilogue of one column half of a QKV tile (8 chunks of 16 tokens x this warp's 32 columns). The accumulator is
// rounded to bf16 first, as the projection's bf16 output is where the reference's qkv_post starts. Pass 1 reads the
// accumulator once: the per-token sums of squares, and the bf16 values stored to their final place in q / k; the
// accumulator goes back to the MMA warp (`release`) right after its last load, so pass 2 overlaps the next tile's
// main loop. Pass 2 waits for the half's four warps (bounded), and then normalises and rotates this warp's own
// stores in place (8 consecutive dims = 4 RoPE pairs per 16-byte vector, read back from L2). Returns false when
// the sums' wait ran out.
template <typename Release>
__device__ __forceinline__ bool qkv_half(const Params& p, uint32_t tbase, uint8_t* epi_stage, int ew, int lane, int q,
                                         int h, int wt, int64_t xb, uint64_t* rms_bar, uint32_t& rms_uses,
                                         volatile int* abort, Release release) {
  constexpr int NC = BN / 2 / kChunk;
  uint8_t* st = epi_stage + ew * kEpiStageBytes;
  const int H = p.qkv_H, Hkv = p.qkv_Hkv;
  const int kind = wt < H ? 0 : (wt < H + Hkv ? 1 : 2);            // q, k or v head
  const int head = wt - (kind == 0 ? 0 : (kind == 1 ? H : H + Hkv));
  const int dim = 32 * q + lane;
  uint32_t r[kChunk];
  if (kind == 2) {   // v: column `dim` of the head, 16 consecutive tokens = 32 contiguous bytes of vt's row
#pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      RL_TMEM_LD16(tbase + c * kChunk, r);
      tmem_ld_wait_regs(r);
      if (c == NC - 1) release();
      const int64_t tok0 = xb + c * kChunk;
      if (tok0 < p.ldv) {   // rows past M are the zero rows of X: zero values, as the padding wants
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w[i]) : "f"(__uint_as_float(r[2 * i + 1])),
              "f"(__uint_as_float(r[2 * i])));
        uint4* dst = reinterpret_cast<uint4*>(p.vt_out + (static_cast<int64_t>(head) * 128 + dim) * p.ldv + tok0);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
    return true;
  }
  uint16_t* out = (kind == 0 ? p.q_out : p.k_out) + static_cast<int64_t>(head) * p.M * 128;
  const int pb = kQkvPartOff + 512 * static_cast<int>(rms_uses & 1u);
  float* part = reinterpret_cast<float*>(st + pb);
  uint16_t* s16 = reinterpret_cast<uint16_t*>(st);
  // pass 1: bf16 values to out (through the staging buffer: 16 tokens x this warp's 64 bytes per chunk), and
  // per-token sums of squares over this warp's 32 columns into its staging buffer
#pragma unroll 1
  for (int c = 0; c < NC; ++c) {
    RL_TMEM_LD16(tbase + c * kChunk, r);
    tmem_ld_wait_regs(r);
    if (c == NC - 1) release();
    float v[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const uint32_t b = float_to_bf16_bits(__uint_as_float(r[j]));
      const float x = bf16_bits_to_float(b);
      v[j] = x * x;
      s16[j * 32 + lane] = static_cast<uint16_t>(b);
    }
    const float ss = warp_sum16(v, lane);
    if (!(lane & 1)) part[c * kChunk + ((lane >> 1) & 15)] = ss;
    __syncwarp();
    const int64_t tok0 = xb + c * kChunk;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = lane + 32 * i, rr = idx >> 2, g = idx & 3;
      const int64_t tok = tok0 + rr;
      if (tok < p.M)
        *reinterpret_cast<uint4*>(out + tok * 128 + 32 * q + g * 8) = reinterpret_cast<const uint4*>(s16 + rr * 32)[g];
    }
    __syncwarp();
  }
  if (lane == 0) mbar_arrive(&rms_bar[h]);   // release: this warp's sums (and its stores) before the others read
  if (!mbar_wait(&rms_bar[h], rms_uses & 1u, abort)) return false;
  ++rms_uses;
  // 1 / rms of the half's 128 tokens from the four warps' sums (each warp its own copy)
  float* rstd = reinterpret_cast<float*>(st + kQkvRstdOff);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int tok = lane + 32 * i;
    float sum = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      sum += reinterpret_cast<const float*>(epi_stage + (4 * h + e) * kEpiStageBytes + pb)[tok];
    rstd[tok] = 1.0f / sqrtf(sum * (1.0f / 128.0f) + 1e-6f);
  }
  __syncwarp();
  // pass 2: lane (t = lane / 4, g = lane % 4) takes dims 32q + 8g .. + 7 of tokens t, t + 8, ...: n = x * rstd * w,
  // then (n0 cos - n1 sin, n0 sin + n1 cos) per pair, the expressions of the separate rl_qkv_post kernel
  const int g = lane & 3, t0 = lane >> 2;
  const float* wsrc = (kind == 0 ? p.w_q : p.w_k) + 32 * q + 8 * g;
  const float4 wa = __ldg(reinterpret_cast<const float4*>(wsrc)), wb = __ldg(reinterpret_cast<const float4*>(wsrc) + 1);
  const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll 1
  for (int k0 = 0; k0 < BN / 2; k0 += 8 * kQkvU) {   // kQkvU tokens per lane per round, their loads issued together
    uint4 xv[kQkvU];
    float4 ca[kQkvU], cb[kQkvU];
#pragma unroll
    for (int u = 0; u < kQkvU; ++u) {
      const int64_t tok = xb + k0 + 8 * u + t0;
      if (tok < p.M) {
        xv[u] = __ldcg(reinterpret_cast<const uint4*>(out + tok * 128 + 32 * q + 8 * g));
        const float4* cs = reinterpret_cast<const float4*>(p.rope_cs + tok * 128 + 32 * q + 8 * g);
        ca[u] = __ldg(cs);
        cb[u] = __ldg(cs + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < kQkvU; ++u) {
      const int tl = k0 + 8 * u + t0;
      const int64_t tok = xb + tl;
      if (tok < p.M) {
        const float inv = rstd[tl];
        const uint32_t xw[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
        const float cc[8] = {ca[u].x, ca[u].y, ca[u].z, ca[u].w, cb[u].x, cb[u].y, cb[u].z, cb[u].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float n0 = __uint_as_float(xw[j] << 16) * inv * w8[2 * j];
          const float n1 = __uint_as_float(xw[j] & 0xFFFF0000u) * inv * w8[2 * j + 1];
          const float co = cc[2 * j], si = cc[2 * j + 1];
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[j]) : "f"(n0 * si + n1 * co), "f"(n0 * co - n1 * si));
        }
        *reinterpret_cast<uint4*>(out + tok * 128 + 32 * q + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  return true;
}

// Expander step shared by both kernels: decode this thread's weight column `row` of the 8 / P eight-deep blocks of
// part `part` of a native W9 tile into bf16 pairs (words[4 * b + i] = K rows 8(part * 8 / P + b) + 2i, +1).
template <int P>
__device__ __forceinline__ void expand_w9(const uint8_t* w9, int row, int part, uint32_t (&words)[32 / P]) {
  constexpr int BPP = 8 / P;
  const uint2 ex = *reinterpret_cast<const uint2*>(w9 + 8192 + row * 8);
  uint4 mq[BPP / 2];
#pragma unroll
  for (int j = 0; j < BPP / 2; ++j)
    mq[j] = *reinterpret_cast<const uint4*>(w9 + ((part * (BPP / 2) + j) * 128 + row) * 16);
#pragma unroll
  for (int b = 0; b < BPP; ++b) {
    const int bk = part * BPP + b;
    const uint32_t E = __byte_perm(bk < 4 ? ex.x : ex.y, 0u, 0x4440u + (bk & 3));
    const uint32_t u0 = (b & 1) ? mq[b >> 1].z : mq[b >> 1].x;
    const uint32_t u1 = (b & 1) ? mq[b >> 1].w : mq[b >> 1].y;
    uint32_t w[4];
    bfp16_decode_block_ob(E, u0, u1, w);
#pragma unroll
    for (int i = 0; i < 4; ++i) words[b * 4 + i] = w[i];
  }
}

// Store decoded words as row `row` of a 128 x 64 bf16 A tile in the 128-byte-swizzled K-major layout, then make the
// writes visible to the tensor cores (async proxy).
template <int P>
__device__ __forceinline__ void store_a_sw128(uint8_t* a_tile, int row, int part, const uint32_t (&words)[32 / P]) {
  constexpr int BPP = 8 / P;
  uint8_t* we = a_tile + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
  for (int b = 0; b < BPP; ++b) {
    const int bk = part * BPP + b;
    *reinterpret_cast<uint4*>(we + ((bk ^ (row & 7)) << 4)) =
        make_uint4(words[b * 4], words[b * 4 + 1], words[b * 4 + 2], words[b * 4 + 3]);
  }
  fence_proxy_async_smem();
}

// E = 1: the QKV epilogue (QK-RMSNorm + RoPE, V transposed; Params::qkv_H) instead of the plain / SwiGLU stores.
template <int V, int S, int G, int P, int E = 0>
__global__ void __launch_bounds__(Cfg<V, S, G, P>::kThreads, 1)
    bfp16_linear_kernel(const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  using C = Cfg<V, S, G, P>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + C::kEpiOff;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + C::kBarOff);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  auto stage_x = [&](int s) { return smem + C::kXOff + s * X_BYTES; };
  auto stage_we = [&](int s) { return smem + C::kWEOff + s * WE_BYTES; };
  auto stage_w9 = [&](int s) { return smem + C::kW9Off + s * W9_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->expf[s], 4 * P);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accf[b], 1);
      mbar_init(&bars->acce[b], C::kEpiWarps);
    }
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->rms[0], 4);
    mbar_init(&bars->rms[1], 4);
    bars->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const int KT = p.KT;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int kiter = 0;
      uint32_t issued = 0, last_par = 0;  // per-stage bit masks (error-path drain)
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int xt = tile % p.num_x_tiles, wt = tile / p.num_x_tiles;
        const uint8_t* wsrc = p.w9 + static_cast<int64_t>(wt) * KT * W9_BYTES;
        for (int kt = 0; kt < KT; ++kt, ++kiter) {
          const int s = kiter % C::kStages;
          const uint32_t ph = (kiter / C::kStages) & 1;
          if (!mbar_wait(&bars->empty[s], ph ^ 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->full[s], X_BYTES + W9_BYTES);
          if (p.conv_W) {   // two 128-pixel runs make the 256-row tile (the second lands 128 rows = 16 KB later)
            load_conv_rows(stage_x(s), &tmap_x, &bars->full[s], p, kt, xt * BN);
            load_conv_rows(stage_x(s) + 128 * 128, &tmap_x, &bars->full[s], p, kt, xt * BN + 128);
          } else {
            tma_load_2d(stage_x(s), &tmap_x, &bars->full[s], kt * BK, xt * BN);
          }
          bulk_load(stage_w9(s), wsrc + static_cast<int64_t>(kt) * W9_BYTES, W9_BYTES, &bars->full[s]);
          issued |= 1u << s;
          last_par = (last_par & ~(1u << s)) | (ph << s);
        }
      }
      if (!ok) {  // let copies already in flight land before the CTA can exit
        for (int s = 0; s < C::kStages; ++s)
          if (issued & (1u << s)) mbar_drain(&bars->full[s], (last_par >> s) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop, one elected lane issues ----------------
    constexpr uint32_t idesc = idesc_bf16(BM, BN);
    int kiter = 0, it = 0;
    bool ok = true, any = false;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int b = (C::kAccBufs == 2) ? (it & 1) : 0;
      const int use = (C::kAccBufs == 2) ? (it >> 1) : it;
      if (!mbar_wait_warp(&bars->acce[b], (use & 1) ^ 1, abort)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem + b * 256;
      for (int kt = 0; kt < KT; ++kt, ++kiter) {
        const int s = kiter % C::kStages;
        const uint32_t ph = (kiter / C::kStages) & 1;
        if (!mbar_wait_warp(&bars->full[s], ph, abort) || !mbar_wait_warp(&bars->expf[s], ph, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(stage_x(s)));
        if (elect_one()) {
          if constexpr (V == kSmemA) {
            const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(stage_we(s)));
#pragma unroll
            for (int k = 0; k < BK / UK; ++k)
              umma_ss(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kt | k) ? 1u : 0u);
          } else {
            const uint32_t a_tmem = tmem + C::kTmemACol + s * (BK / 2);
#pragma unroll
            for (int k = 0; k < BK / UK; ++k)
              umma_ts(d_tmem, a_tmem + k * (UK / 2), bdesc + 2 * k, idesc, (kt | k) ? 1u : 0u);
          }
          umma_commit(&bars->empty[s]);
        }
        __syncwarp();
        any = true;
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&bars->accf[b]);
      __syncwarp();
    }
    if (!ok && any) {  // no MMA may still be reading TMEM / shared memory when the CTA exits
      if (elect_one()) {
        umma_commit(&bars->drain);
        mbar_drain(&bars->drain, 0);
      }
      __syncwarp();
    }
  } else if (warp < C::kEpiWarp0) {
    // ---------------- expanders: W9 (bfp16) -> bf16 A operand ----------------
    constexpr int BPP = 8 / P;                 // 8-deep blocks per part
    const int e = warp - 2;
    const int q = warp & 3;                    // TMEM lane quarter this warp may access
    const int row = 32 * q + lane;             // weight column within the tile
    const int part = (e >> 2) % P;             // which blocks of the stage
    const int grp = (e >> 2) / P;              // which stages: kiter % G == grp
    int kiter = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      for (int kt = 0; kt < KT; ++kt, ++kiter) {
        if (G > 1 && (kiter % G) != grp) continue;
        const int s = kiter % C::kStages;
        const uint32_t ph = (kiter / C::kStages) & 1;
        if (!mbar_wait(&bars->full[s], ph, abort)) { ok = false; break; }
        uint32_t words[4 * BPP];
        expand_w9<P>(stage_w9(s), row, part, words);
        if constexpr (V == kSmemA) {
          store_a_sw128<P>(stage_we(s), row, part, words);
        } else {
          tc_fence_after();
          const uint32_t taddr = tmem + C::kTmemACol + s * (BK / 2) + part * (BK / 2 / P) + ((32u * q) << 16);
          if constexpr (P == 1) {
            RL_TMEM_ST32(taddr, words);
          } else {
            RL_TMEM_ST16(taddr, words);
          }
          tmem_st_wait_regs(words);
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->expf[s]);
      }
    }
  } else {
    // ---------------- epilogue: 8 warps, (lane quarter q, column half h) each ----------------
    const int ew = warp - C::kEpiWarp0;
    const int q = warp & 3;
    const int h = ew >> 2;                         // activation-row half of the tile: columns [128h, 128h + 128)
    const int row = 32 * q + lane;                 // weight column within the tile (native order)
    uint8_t* st = epi_stage + ew * kEpiStageBytes;
    constexpr int NC = BN / 2 / kChunk;            // 8 chunks of 16 columns per warp
    int it = 0;
    bool ok = true;
    [[maybe_unused]] uint32_t rms_uses = 0;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
      const int xt = tile % p.num_x_tiles, wt = tile / p.num_x_tiles;
      const int b = (C::kAccBufs == 2) ? (it & 1) : 0;
      const int use = (C::kAccBufs == 2) ? (it >> 1) : it;
      float bias_v = 0.0f;
      if (p.bias) {
        // native row -> output column (SwiGLU permutes rows inside the tile)
        int col = row;
        if (p.epilogue == RL_EPI_SWIGLU) col = (lane < 16 ? 0 : 64) + 16 * q + (lane & 15);
        bias_v = bf16_bits_to_float(p.bias[static_cast<int64_t>(wt) * BM + col]);
      }
      if (!mbar_wait(&bars->accf[b], use & 1, abort)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tbase = tmem + b * 256 + h * (BN / 2) + ((32u * q) << 16);
      const int64_t xb = static_cast<int64_t>(xt) * BN + h * (BN / 2);
      if constexpr (E == 1) {
        static_assert(C::kAccBufs == 1, "the QKV epilogue's sums are double-buffered for one accumulator");
        if (!qkv_half(p, tbase, epi_stage, ew, lane, q, h, wt, xb, bars->rms, rms_uses, abort, [&] {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars->acce[b]);
            })) {
          ok = false;
          break;
        }
        continue;
      }
      // chunk by chunk: the tcgen05.ld of chunk c+1 is in flight while chunk c is converted and stored
      uint32_t ra[kChunk], rb[kChunk];
      RL_TMEM_LD16(tbase, ra);
      tmem_ld_wait_regs(ra);
#pragma unroll 1
      for (int c = 0; c < NC; c += 2) {
        RL_TMEM_LD16(tbase + (c + 1) * kChunk, rb);
        epilogue_chunk(p, ra, st, lane, q, wt, xb + c * kChunk, bias_v);
        tmem_ld_wait_regs(rb);
        if (c + 2 < NC) {
          RL_TMEM_LD16(tbase + (c + 2) * kChunk, ra);
        } else {  // every column of D is in registers: hand the accumulator back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->acce[b]);
        }
        epilogue_chunk(p, rb, st, lane, q, wt, xb + (c + 1) * kChunk, bias_v);
        if (c + 2 < NC) tmem_ld_wait_regs(ra);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ============================================================================================================
// 2-SM variant: a cluster of two CTAs on neighbouring SMs computes a 256-weight-column x 256-activation-row tile
// with tcgen05.mma.cta_group::2 (M 256 = 128 weight columns per CTA, N 256 = 128 activation rows per CTA). Each CTA
// loads only its half of the activation tile, which halves the L2 -> SM activation traffic per FLOP, and decodes
// its own 128-column weight tile into shared memory (the MMA's A operand, SS form), so the accumulator can be
// double-buffered in TMEM (2 x 256 columns) and the epilogue of tile i overlaps the MMAs of tile i+1.
// Signals: each CTA's loads complete on its own `full` barrier; both CTAs' expanders arrive on the leader's `expf`
// (8 P arrivals per stage) and both CTAs' epilogues on the leader's `acce`; the leader's MMA commits arrive on the
// `empty` / `accf` barriers of both CTAs.
// ============================================================================================================
namespace pair {

constexpr int XH_BYTES = 128 * BK * 2;  // 16384: this CTA's half of the activation tile

// V = kSmemA: decoded weights in shared memory (SS MMA), accumulator double-buffered in TMEM (2 x 256 columns).
// V = kTmemA: decoded weights in TMEM (TS MMA, 32 columns per stage after a single 256-column accumulator), which
//             frees 16 KB of shared memory per stage for a deeper pipeline.
template <int V, int S, int G, int P>
struct Cfg {
  static constexpr int kExpWarps = 4 * P * G;
  static constexpr int kEpiWarps = 8;
  static constexpr int kWarps = 2 + kExpWarps + kEpiWarps;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kEpiWarp0 = 2 + kExpWarps;
  static constexpr int kXOff = 0;                                            // S x 16 KB
  static constexpr int kAOff = kXOff + S * XH_BYTES;                         // SS: S x 16 KB (SW128 K-major)
  static constexpr int kW9Off = kAOff + (V == kSmemA ? S * WE_BYTES : 0);    // S x 9216 B
  static constexpr int kEpiOff = kW9Off + S * W9_BYTES;
  static constexpr int kBarOff = kEpiOff + kEpiWarps * kEpiStageBytes;
  static constexpr int kAccBufs = V == kSmemA ? 2 : 1;
  static constexpr int kTmemACol = 256;                                      // TS: A stages after the accumulator
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kBarOff + 256;
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(V == kSmemA || 256 + S * (BK / 2) <= 512, "TMEM: accumulator + A stages");
  static_assert(S <= 8 && G >= 1 && G <= 4 && (P == 1 || P == 2), "config");
  // A decoder group takes the stages s with s % G == its group, so that it waits on every phase of those stages'
  // load barriers in turn. With S % G != 0 a group would return to a stage only every lcm(S, G) K steps, and its
  // parity wait could be satisfied by a phase two behind the one it needs when a later load lands first.
  static_assert(S % G == 0, "the decoder groups must own whole stages");
};

// Pair tile tt -> (activation tile xt, weight pair wp). Tiles walk groups of p.group_x activation tiles (one group
// when 0); inside a group the activation tile runs fastest, so the clusters in flight share a few weight pairs and
// the group's rows of X stay in L2 while every weight pair streams past them once per group.
__device__ __forceinline__ void pair_tile_coords(const Params& p, int tt, int npairs, int& xt, int& wp) {
  const int gsz = p.group_x > 0 ? p.group_x : p.num_x_tiles;
  const int per_group = gsz * npairs;
  const int g = tt / per_group;
  const int r = tt - g * per_group;
  const int x0 = g * gsz;
  const int gx = min(gsz, p.num_x_tiles - x0);
  wp = r / gx;
  xt = x0 + (r - wp * gx);
}

// E = 1: the QKV epilogue (QK-RMSNorm + RoPE, V transposed; Params::qkv_H) instead of the plain / SwiGLU stores.
template <int V, int S, int G, int P, int E = 0>
__global__ void __launch_bounds__(Cfg<V, S, G, P>::kThreads, 1)
    bfp16_linear_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  using C = Cfg<V, S, G, P>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + C::kEpiOff;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + C::kBarOff);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();          // 0 = leader: issues the pair's MMAs
  const int cid = static_cast<int>(blockIdx.x >> 1), ncl = static_cast<int>(gridDim.x >> 1);
  const int npairs = p.num_w_tiles / 2;
  const int ntiles = p.num_x_tiles * npairs;
  // work items: (pair tile, K range); with p.splits > 1 each item covers KT / p.splits K steps and writes an fp32
  // partial that a reduction kernel adds up
  const int nitems = ntiles * p.splits;

  auto stage_x = [&](int s) { return smem + C::kXOff + s * XH_BYTES; };
  auto stage_a = [&](int s) { return smem + C::kAOff + s * WE_BYTES; };
  auto stage_w9 = [&](int s) { return smem + C::kW9Off + s * W9_BYTES; };
  auto at_leader = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 0); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->expf[s], 2 * 4 * P);        // one expander group of each CTA
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accf[b], 1);
      mbar_init(&bars->acce[b], 2 * C::kEpiWarps);  // the epilogue warps of both CTAs
    }
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->rms[0], 4);
    mbar_init(&bars->rms[1], 4);
    bars->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 0) {
    tmem_alloc_pair(&bars->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers and TMEM exist before any signal crosses the pair
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const int KT = p.KT, KTs = p.KT / p.splits;

  if (warp == 0) {
    // ---------------- producer: this CTA's activation half and weight tile ----------------
    if (lane == 0) {
      int kiter = 0;
      uint32_t issued = 0, last_par = 0;
      bool ok = true;
      for (int t = cid; ok && t < nitems; t += ncl) {
        const int tt = t % ntiles, kt0 = (t / ntiles) * KTs;
        int xt, wp;
        pair_tile_coords(p, tt, npairs, xt, wp);
        const int wt = 2 * wp + static_cast<int>(rank);
        const uint8_t* wsrc = p.w9 + static_cast<int64_t>(wt) * KT * W9_BYTES;
        for (int kt = kt0; kt < kt0 + KTs; ++kt, ++kiter) {
          const int s = kiter % S;
          const uint32_t ph = (kiter / S) & 1;
          if (!mbar_wait(&bars->empty[s], ph ^ 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->full[s], XH_BYTES + W9_BYTES);
          if (p.conv_W)
            load_conv_rows(stage_x(s), &tmap_x, &bars->full[s], p, kt, xt * BN + static_cast<int>(rank) * 128);
          else
            tma_load_2d(stage_x(s), &tmap_x, &bars->full[s], kt * BK, xt * BN + static_cast<int>(rank) * 128);
          bulk_load(stage_w9(s), wsrc + static_cast<int64_t>(kt) * W9_BYTES, W9_BYTES, &bars->full[s]);
          issued |= 1u << s;
          last_par = (last_par & ~(1u << s)) | (ph << s);
        }
      }
      if (!ok) {
        for (int s = 0; s < S; ++s)
          if (issued & (1u << s)) mbar_drain(&bars->full[s], (last_par >> s) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA): warp-wide loop, elected lane issues ----------------
    if (rank == 0) {
      constexpr uint32_t idesc = idesc_bf16(2 * BM, BN);
      int kiter = 0, it = 0;
      bool ok = true, any = false;
      for (int t = cid; ok && t < nitems; t += ncl, ++it) {
        const int b = C::kAccBufs == 2 ? (it & 1) : 0, use = C::kAccBufs == 2 ? (it >> 1) : it;
        if (!mbar_wait_warp(&bars->acce[b], (use & 1) ^ 1, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + b * 256;
        for (int kt = 0; kt < KTs; ++kt, ++kiter) {   // kt: K step within the item (accumulate from its second)
          const int s = kiter % S;
          const uint32_t ph = (kiter / S) & 1;
          // both CTAs' expanders have decoded stage s, which they did after its loads landed
          if (!mbar_wait_warp(&bars->expf[s], ph, abort)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(stage_x(s)));
          if (elect_one()) {
            if constexpr (V == kSmemA) {
              const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(stage_a(s)));
#pragma unroll
              for (int k = 0; k < BK / UK; ++k)
                umma_ss_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kt | k) ? 1u : 0u);
            } else {
              const uint32_t a_tmem = tmem + C::kTmemACol + s * (BK / 2);
#pragma unroll
              for (int k = 0; k < BK / UK; ++k)
                umma_ts_pair(d_tmem, a_tmem + k * (UK / 2), bdesc + 2 * k, idesc, (kt | k) ? 1u : 0u);
            }
            umma_commit_pair(mapa_shared(smem_u32(&bars->empty[s]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&bars->empty[s]), 1));
          }
          __syncwarp();
          any = true;
        }
        if (!ok) break;
        if (elect_one()) {
          umma_commit_pair(mapa_shared(smem_u32(&bars->accf[b]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&bars->accf[b]), 1));
        }
        __syncwarp();
      }
      if (!ok && any) {  // no MMA may still be reading shared memory or TMEM when the CTAs exit
        if (elect_one()) {
          umma_commit_pair(mapa_shared(smem_u32(&bars->drain), 0));
          mbar_drain(&bars->drain, 0);
        }
        __syncwarp();
      }
    }
  } else if (warp < C::kEpiWarp0) {
    // ---------------- expanders: this CTA's W9 tile -> bf16 A tile in shared memory ----------------
    constexpr int BPP = 8 / P;
    const int e = warp - 2;
    const int row = 32 * (warp & 3) + lane;
    const int part = (e >> 2) % P;
    const int grp = (e >> 2) / P;
    int kiter = 0;
    bool ok = true;
    for (int t = cid; ok && t < nitems; t += ncl) {
      for (int kt = 0; kt < KTs; ++kt, ++kiter) {
        if (G > 1 && (kiter % G) != grp) continue;
        const int s = kiter % S;
        const uint32_t ph = (kiter / S) & 1;
        if (!mbar_wait(&bars->full[s], ph, abort)) { ok = false; break; }
        uint32_t words[4 * BPP];
        expand_w9<P>(stage_w9(s), row, part, words);
        if constexpr (V == kSmemA) {
          store_a_sw128<P>(stage_a(s), row, part, words);
        } else {
          tc_fence_after();
          const uint32_t taddr = tmem + C::kTmemACol + s * (BK / 2) + part * (BK / 2 / P) + ((32u * (warp & 3)) << 16);
          if constexpr (P == 1) {
            RL_TMEM_ST32(taddr, words);
          } else {
            RL_TMEM_ST16(taddr, words);
          }
          tmem_st_wait_regs(words);
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(at_leader(&bars->expf[s]));
      }
    }
  } else {
    // ---------------- epilogue: 8 warps, (lane quarter q, column half h) each ----------------
    const int ew = warp - C::kEpiWarp0;
    const int q = warp & 3;
    const int h = ew >> 2;
    const int row = 32 * q + lane;
    uint8_t* st = epi_stage + ew * kEpiStageBytes;
    constexpr int NC = BN / 2 / kChunk;
    int it = 0;
    bool ok = true;
    uint32_t rms_uses = 0;
    for (int t = cid; ok && t < nitems; t += ncl, ++it) {
      const int tt = t % ntiles;
      const int64_t out_off = static_cast<int64_t>(t / ntiles) * p.split_stride;
      int xt, wp;
      pair_tile_coords(p, tt, npairs, xt, wp);
      const int wt = 2 * wp + static_cast<int>(rank);
      const int b = C::kAccBufs == 2 ? (it & 1) : 0, use = C::kAccBufs == 2 ? (it >> 1) : it;
      float bias_v = 0.0f;
      if (p.bias) {
        int col = row;
        if (p.epilogue == RL_EPI_SWIGLU) col = (lane < 16 ? 0 : 64) + 16 * q + (lane & 15);
        bias_v = bf16_bits_to_float(p.bias[static_cast<int64_t>(wt) * BM + col]);
      }
      if (!mbar_wait(&bars->accf[b], use & 1, abort)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tbase = tmem + b * 256 + h * (BN / 2) + ((32u * q) << 16);
      const int64_t xb = static_cast<int64_t>(xt) * BN + h * (BN / 2);
      if constexpr (E == 1) {
        if (!qkv_half(p, tbase, epi_stage, ew, lane, q, h, wt, xb, bars->rms, rms_uses, abort, [&] {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_remote(at_leader(&bars->acce[b]));
            })) {
          ok = false;
          break;
        }
        continue;
      }
      uint32_t ra[kChunk], rb[kChunk];
      RL_TMEM_LD16(tbase, ra);
      tmem_ld_wait_regs(ra);
#pragma unroll 1
      for (int c = 0; c < NC; c += 2) {
        RL_TMEM_LD16(tbase + (c + 1) * kChunk, rb);
        epilogue_chunk(p, ra, st, lane, q, wt, xb + c * kChunk, bias_v, out_off);
        tmem_ld_wait_regs(rb);
        if (c + 2 < NC) {
          RL_TMEM_LD16(tbase + (c + 2) * kChunk, ra);
        } else {  // all of buffer b is in registers: release it to the leader's MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(at_leader(&bars->acce[b]));
        }
        epilogue_chunk(p, rb, st, lane, q, wt, xb + (c + 1) * kChunk, bias_v, out_off);
        if (c + 2 < NC) tmem_ld_wait_regs(ra);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while its peer may still signal its barriers or read its shared memory
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace pair

static int g_variant = 0;  // 0 = default

// Tensor map over X (M x K bf16, row-major) with boxes of 64 K x box_rows rows, 128-byte swizzle.
inline int make_x_map(CUtensorMap* map, const uint16_t* x, int64_t M, int64_t K, int box_rows) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(RL_ERR_CUDA, "rl_linear_bfp16: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult cr = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), gdim, gstride, box,
                          estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(RL_ERR_CUDA, "rl_linear_bfp16: cuTensorMapEncodeTiled failed (%d)", (int)cr);
  return RL_OK;
}

// The A operand's map: 2-D (K, M) with `box_rows` rows, or in conv mode the 3-D map over the (H, W, C) image
// (box = 64 channels x 128 pixels x 1 row; out-of-range elements read as zero).
inline int make_a_map(CUtensorMap* map, const uint16_t* x, const Params& p, int box_rows) {
  if (!p.conv_W) return make_x_map(map, x, p.M, p.K, box_rows);
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(RL_ERR_CUDA, "rl_conv2d_bfp16: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t gdim[3] = {static_cast<cuuint64_t>(p.conv_C), static_cast<cuuint64_t>(p.conv_W),
                              static_cast<cuuint64_t>(p.conv_H)};
  const cuuint64_t gstride[2] = {static_cast<cuuint64_t>(p.conv_C) * 2,
                                 static_cast<cuuint64_t>(p.conv_C) * 2 * static_cast<cuuint64_t>(p.conv_W)};
  const cuuint32_t box[3] = {BK, 128, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult cr = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(x), gdim, gstride, box,
                          estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(RL_ERR_CUDA, "rl_conv2d_bfp16: cuTensorMapEncodeTiled failed (%d)", (int)cr);
  return RL_OK;
}

template <int V, int S, int G, int P, int E = 0>
int launch(const uint16_t* x, const Params& p, cudaStream_t stream) {
  using C = Cfg<V, S, G, P>;
  CUtensorMap tmap;
  int st = make_a_map(&tmap, x, p, BN);
  if (st != RL_OK) return st;
  static bool attr_set[64] = {false};
  int dev = 0;
  RL_TRY_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    RL_TRY_CUDA(cudaFuncSetAttribute(bfp16_linear_kernel<V, S, G, P, E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::kSmemBytes));
    attr_set[dev] = true;
  }
  const int grid = p.num_tiles < sm_count() ? p.num_tiles : sm_count();
  bfp16_linear_kernel<V, S, G, P, E><<<grid, C::kThreads, C::kSmemBytes, stream>>>(tmap, p);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

// How many 2-CTA clusters of the pair kernel can be resident at once on the current device (cached per device). A
// cluster's two CTAs share a GPC, so this depends on the chip's GPC layout, not only on the SM count.
template <int V, int S, int G, int P, int E = 0>
int pair_max_clusters(int* out) {
  using C = pair::Cfg<V, S, G, P>;
  auto kernel = pair::bfp16_linear_pair_kernel<V, S, G, P, E>;
  static int cached[64] = {0};
  int dev = 0;
  RL_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(RL_ERR_CUDA, "rl_linear_bfp16: device index %d", dev);
  if (cached[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2);
    RL_TRY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    int n = 0;
    RL_TRY_CUDA(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
    if (n <= 0) return fail(RL_ERR_UNSUPPORTED, "rl_linear_bfp16: no CTA pair fits on this device");
    cached[dev] = n;
  }
  *out = cached[dev];
  return RL_OK;
}

// Pair kernel: clusters of two CTAs; the grid is as many clusters as can be resident at once (at most one per pair
// tile), each walking pair tiles with stride = number of clusters.
template <int V, int S, int G, int P, int E = 0>
int launch_pair(const uint16_t* x, const Params& p, cudaStream_t stream) {
  using C = pair::Cfg<V, S, G, P>;
  auto kernel = pair::bfp16_linear_pair_kernel<V, S, G, P, E>;
  CUtensorMap tmap;
  int st = make_a_map(&tmap, x, p, 128);
  if (st != RL_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  int st2 = pair_max_clusters<V, S, G, P, E>(&max_clusters);
  if (st2 != RL_OK) return st2;
  const int ntiles = p.num_x_tiles * (p.num_w_tiles / 2) * p.splits;
  const int nclusters = ntiles < max_clusters ? ntiles : max_clusters;
  cfg.gridDim = dim3(2 * nclusters);
  RL_TRY_CUDA(cudaLaunchKernelEx(&cfg, kernel, tmap, p));
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

// Kernel variants selectable with rl_set_gemm_variant (code = 1000 * P + 100 * G + 10 * V + S; V = 1 / 2: the 1-SM
// kernel with A in shared memory / TMEM, V = 3 / 4: the 2-SM pair kernel with A in shared memory / TMEM; every code
// has S % G == 0). 0 = default: the pair kernel with A in TMEM (8 stages, decode split in two parts x two groups)
// when N is a multiple of 256, else the 1-SM kernel with A in TMEM (code kDefault1Sm). 1 - 4: one code per kernel
// form for the tests.
constexpr int kDefault1Sm = 2224;
int dispatch(int code, const uint16_t* x, const Params& p, cudaStream_t stream) {
  const bool pairable = p.num_w_tiles % 2 == 0;
  if (code == 0) code = pairable ? 2248 : kDefault1Sm;
  switch (code) {
    case 1:
    case 1313: return launch<kSmemA, 3, 3, 1>(x, p, stream);
    case 1125: return launch<kTmemA, 5, 1, 1>(x, p, stream);
    case 2125: return launch<kTmemA, 5, 1, 2>(x, p, stream);
    case 1224: return launch<kTmemA, 4, 2, 1>(x, p, stream);
    case 2:
    case 2224: return launch<kTmemA, 4, 2, 2>(x, p, stream);
    default: break;
  }
  if (code == 3 || code == 4 || code == 1333 || code == 1234 || code == 1346 || code == 1448 || code == 2248) {
    if (!pairable) return fail(RL_ERR_ARGUMENT, "rl_linear_bfp16: the pair kernel needs N %% 256 == 0");
    switch (code) {
      case 3:
      case 1333: return launch_pair<kSmemA, 3, 3, 1>(x, p, stream);
      case 1234: return launch_pair<kSmemA, 4, 2, 1>(x, p, stream);
      case 1346: return launch_pair<kTmemA, 6, 3, 1>(x, p, stream);
      case 4:
      case 1448: return launch_pair<kTmemA, 8, 4, 1>(x, p, stream);
      default: return launch_pair<kTmemA, 8, 2, 2>(x, p, stream);
    }
  }
  return fail(RL_ERR_ARGUMENT, "rl_linear_bfp16: unknown kernel variant %d", code);
}

// Activation tiles per group of the pair kernel's tile order (pair_tile_coords): groups hold ~40 MB of X, a third of
// the 126 MB L2, and are balanced in size. Every group streams all the weights once, and the clusters in flight read
// the group's X from L2 instead of re-reading X from HBM for every weight pair (M 17408 x K 3072: X alone is 107 MB;
// measured 965 us per launch in groups against 1138 us in one group).
inline int group_tiles(int num_x_tiles, int64_t K) {
  const int64_t gmax = (static_cast<int64_t>(40) << 20) / (static_cast<int64_t>(BN) * K * 2);
  const int64_t cap = gmax < 1 ? 1 : gmax;
  const int64_t groups = (num_x_tiles + cap - 1) / cap;
  return static_cast<int>((num_x_tiles + groups - 1) / groups);
}

// Split-K for the pair kernel on a grid that would not fill the GPU: the largest S in {2, 4} with S x (pair tiles)
// <= the pair kernel's resident clusters (one pair of SMs each), KT % S == 0 and at least 16 K steps per split; 1
// when no split helps (or no device answers the occupancy query).
inline int choose_splits(int64_t M, int64_t K, int64_t N) {
  if (N % 256) return 1;
  int resident = 0;
  if (pair_max_clusters<kTmemA, 8, 2, 2>(&resident) != RL_OK) return 1;
  const int64_t clusters = resident;
  const int64_t tiles = (M + BN - 1) / BN * (N / 256);
  const int64_t KT = K / BK;
  int S = 1;
  for (int c = 2; c <= 4; c *= 2)
    if (tiles * c <= clusters && KT % c == 0 && KT / c >= 16) S = c;
  return S;
}

// out[m][n] = sum over s of part[s][m][n] (+ bias[n]), to bf16 (round to nearest even) or fp32; 4 columns a thread.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ part, int S, int64_t MN, int64_t N,
                                                            const uint16_t* __restrict__ bias, void* __restrict__ out,
                                                            int out_f32) {
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x) * 4; i < MN;
       i += static_cast<int64_t>(gridDim.x) * 256 * 4) {
    float4 a = *reinterpret_cast<const float4*>(part + i);
    for (int sp = 1; sp < S; ++sp) {
      const float4 b = *reinterpret_cast<const float4*>(part + sp * MN + i);
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    if (bias) {
      const int64_t n = i % N;
      a.x += bf16_bits_to_float(bias[n]);
      a.y += bf16_bits_to_float(bias[n + 1]);
      a.z += bf16_bits_to_float(bias[n + 2]);
      a.w += bf16_bits_to_float(bias[n + 3]);
    }
    if (out_f32) {
      *reinterpret_cast<float4*>(static_cast<float*>(out) + i) = a;
    } else {
      const uint32_t lo = float_to_bf16_bits(a.x) | (float_to_bf16_bits(a.y) << 16);
      const uint32_t hi = float_to_bf16_bits(a.z) | (float_to_bf16_bits(a.w) << 16);
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + i) = make_uint2(lo, hi);
    }
  }
}

}  // namespace gemm
}  // namespace rl

extern "C" {

size_t rl_linear_bfp16_workspace(int64_t M, int64_t K, int64_t N, int epilogue) {
  if (M <= 0 || K < 64 || K % 64 || N < 128 || N % 128 || epilogue == RL_EPI_SWIGLU) return 0;
  const int S = rl::gemm::choose_splits(M, K, N);
  return S > 1 ? static_cast<size_t>(S) * M * N * 4 : 0;
}

int rl_linear_bfp16_ws(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                       const uint16_t* bias, int epilogue, void* out, int out_dtype, void* workspace,
                       size_t workspace_bytes, rl_stream_t stream) {
  using namespace rl;
  using namespace rl::gemm;
  const size_t need = rl_linear_bfp16_workspace(M, K, N, epilogue);
  if (need == 0 || g_variant != 0 || workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))
    return rl_linear_bfp16(x, M, K, w_native, N, bias, epilogue, out, out_dtype, stream);
  RL_REQUIRE(epilogue != RL_EPI_BIAS || bias != nullptr, RL_ERR_ARGUMENT, "rl_linear_bfp16: RL_EPI_BIAS needs bias");
  RL_REQUIRE(out_dtype == RL_BF16 || out_dtype == RL_F32, RL_ERR_ARGUMENT, "rl_linear_bfp16: bad out dtype");
  RL_REQUIRE(x && w_native && out, RL_ERR_ARGUMENT, "rl_linear_bfp16: NULL pointer");
  RL_REQUIRE(aligned(x, 16) && aligned(w_native, 16) && aligned(out, 16), RL_ERR_ALIGNMENT,
             "rl_linear_bfp16: x, w_native and out must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_linear_bfp16: needs an sm_100 device");
  Params p;
  p.w9 = w_native;
  p.bias = nullptr;
  p.out = workspace;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out_f32 = 1;
  p.epilogue = RL_EPI_NONE;
  p.num_x_tiles = static_cast<int>((M + BN - 1) / BN);
  p.num_w_tiles = static_cast<int>(N / BM);
  p.num_tiles = p.num_x_tiles * p.num_w_tiles;
  p.KT = static_cast<int>(K / BK);
  p.group_x = group_tiles(p.num_x_tiles, K);
  p.splits = choose_splits(M, K, N);
  p.split_stride = M * N;
  int st = launch_pair<kTmemA, 8, 2, 2>(x, p, stream);
  if (st != RL_OK) return st;
  const int64_t MN = M * N;
  const int64_t blocks = (MN / 4 + 255) / 256, cap = static_cast<int64_t>(sm_count()) * 8;
  splitk_reduce_kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, stream>>>(
      static_cast<const float*>(workspace), p.splits, MN, N, epilogue == RL_EPI_BIAS ? bias : nullptr, out,
      out_dtype == RL_F32 ? 1 : 0);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_gemm_pair_clusters(void) {
  int n = 0;
  return rl::gemm::pair_max_clusters<rl::gemm::kTmemA, 8, 2, 2>(&n) == RL_OK ? n : 0;
}

int rl_set_gemm_variant(int variant) {
  const int prev = rl::gemm::g_variant;
  rl::gemm::g_variant = variant;
  return prev;
}

int rl_linear_bfp16(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                    const uint16_t* bias, int epilogue, void* out, int out_dtype, rl_stream_t stream) {
  return rl_linear_bfp16_mirror(x, M, K, w_native, N, bias, epilogue, out, nullptr, out_dtype, stream);
}

int rl_linear_bfp16_mirror(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                           const uint16_t* bias, int epilogue, void* out, void* mirror, int out_dtype,
                           rl_stream_t stream) {
  using namespace rl;
  using namespace rl::gemm;
  RL_REQUIRE(x && w_native && out, RL_ERR_ARGUMENT, "rl_linear_bfp16: NULL pointer");
  RL_REQUIRE(!mirror || (out_dtype == RL_BF16 && epilogue != RL_EPI_SWIGLU && aligned(mirror, 16)), RL_ERR_ARGUMENT,
             "rl_linear_bfp16_mirror: the mirror needs a 16-byte aligned bf16 output without SwiGLU");
  RL_REQUIRE(M >= 0 && K >= 64 && K % 64 == 0 && N >= 128 && N % 128 == 0, RL_ERR_ARGUMENT,
             "rl_linear_bfp16: need K %% 64 == 0, N %% 128 == 0 (M=%lld K=%lld N=%lld)", (long long)M, (long long)K,
             (long long)N);
  RL_REQUIRE(epilogue == RL_EPI_NONE || epilogue == RL_EPI_BIAS || epilogue == RL_EPI_SWIGLU, RL_ERR_ARGUMENT,
             "rl_linear_bfp16: bad epilogue %d", epilogue);
  RL_REQUIRE(epilogue != RL_EPI_BIAS || bias != nullptr, RL_ERR_ARGUMENT, "rl_linear_bfp16: RL_EPI_BIAS needs bias");
  RL_REQUIRE(out_dtype == RL_BF16 || out_dtype == RL_F32, RL_ERR_ARGUMENT, "rl_linear_bfp16: bad out dtype");
  RL_REQUIRE(epilogue != RL_EPI_SWIGLU || out_dtype == RL_BF16, RL_ERR_ARGUMENT,
             "rl_linear_bfp16: SwiGLU writes bf16 (bfp16-rounded) only");
  RL_REQUIRE(aligned(x, 16) && aligned(w_native, 16) && aligned(out, 16), RL_ERR_ALIGNMENT,
             "rl_linear_bfp16: x, w_native and out must be 16-byte aligned");
  RL_REQUIRE(K <= (int64_t)1 << 31 && M < ((int64_t)1 << 31), RL_ERR_ARGUMENT, "rl_linear_bfp16: size too large");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_linear_bfp16: needs an sm_100 device");
  if (M == 0) return RL_OK;
  Params p;
  p.w9 = w_native;
  p.bias = (epilogue == RL_EPI_NONE) ? nullptr : bias;
  p.out = out;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out_f32 = out_dtype == RL_F32;
  p.epilogue = epilogue;
  p.num_x_tiles = static_cast<int>((M + BN - 1) / BN);
  p.num_w_tiles = static_cast<int>(N / BM);
  p.num_tiles = p.num_x_tiles * p.num_w_tiles;
  p.KT = static_cast<int>(K / BK);
  p.group_x = group_tiles(p.num_x_tiles, K);
  p.splits = 1;
  p.split_stride = 0;
  p.mirror = mirror;
  return dispatch(g_variant, x, p, stream);
}

int rl_qkv_linear(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int H, int Hkv,
                  const float* rope_cs, const float* w_q, const float* w_k, uint16_t* q, uint16_t* k, uint16_t* vt,
                  int64_t ldv, rl_stream_t stream) {
  using namespace rl;
  using namespace rl::gemm;
  RL_REQUIRE(x && w_native && rope_cs && w_q && w_k && q && k && vt, RL_ERR_ARGUMENT, "rl_qkv_linear: NULL pointer");
  RL_REQUIRE(H > 0 && Hkv > 0 && H % Hkv == 0 && M >= 0 && K >= 64 && K % 64 == 0, RL_ERR_ARGUMENT,
             "rl_qkv_linear: need H, Hkv > 0, H %% Hkv == 0, K %% 64 == 0");
  RL_REQUIRE(ldv >= M && ldv % 16 == 0 && ldv <= (M + BN - 1) / BN * BN, RL_ERR_ARGUMENT,
             "rl_qkv_linear: need M <= ldv <= M rounded up to 256, ldv %% 16 == 0 (M=%lld ldv=%lld)", (long long)M,
             (long long)ldv);
  RL_REQUIRE(aligned(x, 16) && aligned(w_native, 16) && aligned(rope_cs, 16) && aligned(w_q, 16) && aligned(w_k, 16) &&
                 aligned(q, 16) && aligned(k, 16) && aligned(vt, 16),
             RL_ERR_ALIGNMENT, "rl_qkv_linear: pointers must be 16-byte aligned");
  RL_REQUIRE(K <= (int64_t)1 << 31 && M < ((int64_t)1 << 31), RL_ERR_ARGUMENT, "rl_qkv_linear: size too large");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_qkv_linear: needs an sm_100 device");
  if (M == 0) return RL_OK;
  const int64_t N = static_cast<int64_t>(H + 2 * Hkv) * 128;
  Params p;
  p.w9 = w_native;
  p.bias = nullptr;
  p.out = q;                  // unused: the QKV epilogue writes q, k and vt
  p.M = M;
  p.N = N;
  p.K = K;
  p.out_f32 = 0;
  p.epilogue = RL_EPI_NONE;
  p.num_x_tiles = static_cast<int>((M + BN - 1) / BN);
  p.num_w_tiles = static_cast<int>(N / BM);
  p.num_tiles = p.num_x_tiles * p.num_w_tiles;
  p.KT = static_cast<int>(K / BK);
  p.group_x = group_tiles(p.num_x_tiles, K);
  p.splits = 1;
  p.split_stride = 0;
  p.qkv_H = H;
  p.qkv_Hkv = Hkv;
  p.rope_cs = rope_cs;
  p.w_q = w_q;
  p.w_k = w_k;
  p.q_out = q;
  p.k_out = k;
  p.vt_out = vt;
  p.ldv = ldv;
  // whole 256-column head pairs on the 2-SM pair kernel, else (an odd head count) the 1-SM kernel
  if (p.num_w_tiles % 2 == 0) return launch_pair<kTmemA, 8, 2, 2, 1>(x, p, stream);
  return launch<kTmemA, 4, 2, 2, 1>(x, p, stream);
}

int rl_linear_bfp16_partial(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                            uint16_t* out, uint16_t* mirror, rl_stream_t stream) {
  using namespace rl;
  using namespace rl::gemm;
  RL_REQUIRE(x && w_native && out, RL_ERR_ARGUMENT, "rl_linear_bfp16_partial: NULL pointer");
  RL_REQUIRE(M >= 0 && K >= 64 && K % 64 == 0 && N >= 128 && N % 128 == 0, RL_ERR_ARGUMENT,
             "rl_linear_bfp16_partial: need K %% 64 == 0, N %% 128 == 0 (M=%lld K=%lld N=%lld)", (long long)M,
             (long long)K, (long long)N);
  RL_REQUIRE(aligned(x, 16) && aligned(w_native, 16) && aligned(out, 16) && aligned(mirror, 16), RL_ERR_ALIGNMENT,
             "rl_linear_bfp16_partial: x, w_native, out and mirror must be 16-byte aligned");
  RL_REQUIRE(K <= (int64_t)1 << 31 && M < ((int64_t)1 << 31), RL_ERR_ARGUMENT,
             "rl_linear_bfp16_partial: size too large");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_linear_bfp16_partial: needs an sm_100 device");
  if (M == 0) return RL_OK;
  Params p;
  p.w9 = w_native;
  p.bias = nullptr;
  p.out = out;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out_f32 = 0;
  p.epilogue = RL_EPI_NONE;
  p.num_x_tiles = static_cast<int>((M + BN - 1) / BN);
  p.num_w_tiles = static_cast<int>(N / BM);
  p.num_tiles = p.num_x_tiles * p.num_w_tiles;
  p.KT = static_cast<int>(K / BK);
  p.group_x = group_tiles(p.num_x_tiles, K);
  p.splits = 1;
  p.split_stride = 0;
  p.mirror = mirror;
  p.chunked = 1;
  return dispatch(g_variant, x, p, stream);
}

int rl_linear_bfp16_scatter(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_native, int64_t N,
                            uint16_t* const* dsts, int W, int64_t rows_per_rank, rl_stream_t stream) {
  using namespace rl;
  using namespace rl::gemm;
  RL_REQUIRE(x && w_native && dsts && W >= 1 && W <= 64, RL_ERR_ARGUMENT, "rl_linear_bfp16_scatter: bad arguments");
  RL_REQUIRE(M >= 0 && K >= 64 && K % 64 == 0 && N >= 128 && N % 128 == 0 && rows_per_rank > 0 &&
                 rows_per_rank % 16 == 0 && M == W * rows_per_rank,
             RL_ERR_ARGUMENT,
             "rl_linear_bfp16_scatter: need K %% 64 == 0, N %% 128 == 0, M = W x rows_per_rank, rows_per_rank %% 16 "
             "== 0 (M=%lld K=%lld N=%lld W=%d)",
             (long long)M, (long long)K, (long long)N, W);
  RL_REQUIRE(aligned(x, 16) && aligned(w_native, 16) && aligned(dsts, 8), RL_ERR_ALIGNMENT,
             "rl_linear_bfp16_scatter: x and w_native must be 16-byte aligned");
  RL_REQUIRE(K <= (int64_t)1 << 31 && M < ((int64_t)1 << 31), RL_ERR_ARGUMENT,
             "rl_linear_bfp16_scatter: size too large");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_linear_bfp16_scatter: needs an sm_100 device");
  if (M == 0) return RL_OK;
  Params p;
  p.w9 = w_native;
  p.bias = nullptr;
  p.out = nullptr;
  p.M = M;
  p.N = N;
  p.K = K;
  p.out_f32 = 0;
  p.epilogue = RL_EPI_NONE;
  p.num_x_tiles = static_cast<int>((M + BN - 1) / BN);
  p.num_w_tiles = static_cast<int>(N / BM);
  p.num_tiles = p.num_x_tiles * p.num_w_tiles;
  p.KT = static_cast<int>(K / BK);
  p.group_x = group_tiles(p.num_x_tiles, K);
  p.splits = 1;
  p.split_stride = 0;
  p.chunked = 1;
  p.scatter = dsts;
  p.scatter_rows = rows_per_rank;
  return dispatch(g_variant, x, p, stream);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------------------
// Convolution as an implicit GEMM: the A tile of each K step is loaded straight from the (H, W, C) image.
// ------------------------------------------------------------------------------------------------------------
namespace rl {
namespace gemm {

// out (H * W, N) = conv(x (H, W, C), w) with the weight packed as B = [(dy, dx, c padded to cpt * 64)][N]; needs
// W % 128 == 0 (a 128-pixel A run stays in one image row), C % 8 == 0 and C >= 64 (the 64-channel box never exceeds
// the channel extent as a whole).
int linear_conv(const uint16_t* x, int H, int W, int C, int taps, const uint8_t* w_native, int64_t N,
                const uint16_t* bias, uint16_t* out, cudaStream_t stream) {
  RL_REQUIRE(W % 128 == 0 && C % 8 == 0 && C >= 64 && (taps == 1 || taps == 3), RL_ERR_ARGUMENT,
             "conv: implicit GEMM needs W %% 128 == 0, C %% 8 == 0, C >= 64");
  Params p;
  p.w9 = w_native;
  p.bias = bias;
  p.out = out;
  p.M = static_cast<int64_t>(H) * W;
  p.N = N;
  p.conv_cpt = (C + BK - 1) / BK;
  p.K = static_cast<int64_t>(taps) * taps * p.conv_cpt * BK;
  p.out_f32 = 0;
  p.epilogue = bias ? RL_EPI_BIAS : RL_EPI_NONE;
  p.num_x_tiles = static_cast<int>((p.M + BN - 1) / BN);
  p.num_w_tiles = static_cast<int>(N / BM);
  p.num_tiles = p.num_x_tiles * p.num_w_tiles;
  p.KT = static_cast<int>(p.K / BK);
  p.group_x = group_tiles(p.num_x_tiles, p.K);
  p.splits = 1;
  p.split_stride = 0;
  p.conv_W = W;
  p.conv_H = H;
  p.conv_C = C;
  p.conv_taps = taps;
  // 1-SM shapes: 4 stages, 2 decoder groups, one part (1224) measured 3-5 % faster than the plain-GEMM default on
  // the VAE's 128^2 x 1152 and 512^2 x 288 convolutions (bit-identical results)
  const int code = (g_variant == 0 && p.num_w_tiles % 2 != 0) ? 1224 : g_variant;
  return dispatch(code, x, p, stream);
}

}  // namespace gemm
}  // namespace rl

// ------------------------------------------------------------------------------------------------------------
// SwiGLU MLP: the Qwen3-VL / DiT feed-forward as two packed-weight GEMMs through a caller workspace.
// ------------------------------------------------------------------------------------------------------------
namespace rl {
namespace mlp {

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace layout: [quantised x (M x K bf16) unless x is already bfp16-exact][H (M x F bf16)][split-K partials of
// the down GEMM, sized for N = K (the usual MLP), when the down GEMM's grid is small enough to split (optional: a
// smaller workspace runs the down GEMM unsplit)].
inline size_t base_bytes(int64_t M, int64_t K, int64_t F, int x_quantized) {
  return (x_quantized ? 0 : align256(static_cast<size_t>(M) * K * 2)) + align256(static_cast<size_t>(M) * F * 2);
}
inline size_t workspace_bytes(int64_t M, int64_t K, int64_t F, int x_quantized) {
  return base_bytes(M, K, F, x_quantized) + align256(rl_linear_bfp16_workspace(M, F, K, RL_EPI_NONE));
}

int run(const void* x, int x_dtype, int x_quantized, int64_t M, int64_t K, const uint8_t* w_up, int64_t F2,
        const uint8_t* w_down, int64_t N, void* out, int out_dtype, uint8_t* ws, size_t ws_bytes,
        cudaStream_t stream) {
  RL_REQUIRE(x && w_up && w_down && out && ws, RL_ERR_ARGUMENT, "swiglu_mlp: NULL pointer");
  RL_REQUIRE(F2 % 256 == 0 && K % 64 == 0 && N % 128 == 0 && M >= 0, RL_ERR_ARGUMENT,
             "swiglu_mlp: need K %% 64 == 0, 2F %% 256 == 0, N %% 128 == 0");
  RL_REQUIRE(!x_quantized || x_dtype == RL_BF16, RL_ERR_ARGUMENT, "swiglu_mlp: a quantised x must be bf16");
  const int64_t F = F2 / 2;
  const size_t base = base_bytes(M, K, F, x_quantized);
  RL_REQUIRE(ws_bytes >= base, RL_ERR_ARGUMENT, "swiglu_mlp: workspace of %zu bytes, need at least %zu", ws_bytes, base);
  RL_REQUIRE(aligned(ws, 256), RL_ERR_ALIGNMENT, "swiglu_mlp: workspace must be 256-byte aligned");
  if (M == 0) return RL_OK;
  const uint16_t* xq = static_cast<const uint16_t*>(x);
  uint8_t* h = ws;
  if (!x_quantized) {
    const int st = rl_quantize_bfp16(x, x_dtype, M, K, RL_ROWMAJOR, nullptr, reinterpret_cast<uint16_t*>(ws), stream);
    if (st != RL_OK) return st;
    xq = reinterpret_cast<const uint16_t*>(ws);
    h = ws + align256(static_cast<size_t>(M) * K * 2);
  }
  int st = rl_linear_bfp16(xq, M, K, w_up, F2, nullptr, RL_EPI_SWIGLU, h, RL_BF16, stream);
  if (st != RL_OK) return st;
  return rl_linear_bfp16_ws(reinterpret_cast<const uint16_t*>(h), M, F, w_down, N, nullptr, RL_EPI_NONE, out,
                            out_dtype, ws + base, ws_bytes - base, stream);
}

}  // namespace mlp
}  // namespace rl

extern "C" {

size_t rl_swiglu_mlp_workspace(int64_t M, int64_t K, int64_t F, int x_quantized) {
  return rl::mlp::workspace_bytes(M, K, F, x_quantized);
}

int rl_swiglu_mlp(const void* x, int x_dtype, int x_quantized, int64_t M, int64_t K, const uint8_t* w_up, int64_t F2,
                  const uint8_t* w_down, int64_t N, void* out, int out_dtype, void* workspace,
                  size_t workspace_bytes, rl_stream_t stream) {
  return rl::mlp::run(x, x_dtype, x_quantized, M, K, w_up, F2, w_down, N, out, out_dtype,
                      static_cast<uint8_t*>(workspace), workspace_bytes, stream);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------------------
// SwiGLU MLP without any allocation, for callers that cannot allocate device memory: its scratch is a fixed
// file-scope device array that every GPU loading this library holds until the process exits.
// ------------------------------------------------------------------------------------------------------------
namespace rl {
namespace mlp {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;  // 32 MiB: config 2 (M 512, K 4096, F 12288) needs 16.8 MB

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch, looked up once per device (with that device current). In host code the
// array's name only stands in for the symbol; a kernel must be given this address instead.
static uint8_t* static_scratch_address(int& status) {
  constexpr int kMaxDev = 64;
  static uint8_t* addr[kMaxDev] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    status = fail(RL_ERR_CUDA, "rl_swiglu_mlp_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      status = fail(RL_ERR_CUDA, "rl_swiglu_mlp_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<uint8_t*>(p);
  }
  status = RL_OK;
  return addr[dev];
}

}  // namespace mlp
}  // namespace rl

extern "C" {

size_t rl_swiglu_mlp_noalloc_capacity(void) { return rl::mlp::kStaticScratchBytes; }

int rl_swiglu_mlp_noalloc(const void* x, int x_dtype, int x_quantized, int64_t M, int64_t K, const uint8_t* w_up,
                          int64_t F2, const uint8_t* w_down, int64_t N, void* out, int out_dtype,
                          rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(M >= 0 && K > 0 && F2 > 0 && N > 0, RL_ERR_ARGUMENT, "rl_swiglu_mlp_noalloc: bad shape");
  // bound the sizes before multiplying them, so that the byte count below cannot wrap
  RL_REQUIRE(M < (int64_t(1) << 31) && K <= (int64_t(1) << 31) && F2 <= (int64_t(1) << 31), RL_ERR_ARGUMENT,
             "rl_swiglu_mlp_noalloc: size too large (M=%lld K=%lld 2F=%lld)", (long long)M, (long long)K,
             (long long)F2);
  const size_t need = mlp::base_bytes(M, K, F2 / 2, x_quantized);   // the split-K partials are optional
  RL_REQUIRE(need <= mlp::kStaticScratchBytes, RL_ERR_ARGUMENT,
             "rl_swiglu_mlp_noalloc: M=%lld K=%lld F=%lld needs %zu bytes of scratch, more than the fixed %zu bytes "
             "(use rl_swiglu_mlp with a caller workspace)",
             (long long)M, (long long)K, (long long)(F2 / 2), need, mlp::kStaticScratchBytes);
  int st = RL_OK;
  uint8_t* scratch = mlp::static_scratch_address(st);
  if (!scratch) return st;
  return mlp::run(x, x_dtype, x_quantized, M, K, w_up, F2, w_down, N, out, out_dtype, scratch,
                  mlp::kStaticScratchBytes, stream);
}

}  // extern "C"
