// Row kernels between the GEMMs of a DiT block (HBM-bound, one warp per row):
//   ln_mod   x' = bf16(x + g * branch); y = LayerNorm(x') * sc, rounded to bfp16 along the row (the next GEMM's
//            A operand). Restates kernels/glue/ln_mod.cc (ln_p1 / ln_fin / ln_p2, lines 92-204) and its numpy model
//            redline/run_ln.py:65-71, with g = tanh(gate), sc = 1 + scale picked per row from two parameter rows.
//   qkv_post per head: RMSNorm over 128 dims (eps 1e-6) * w, complex RoPE on adjacent pairs; V passes through and is
//            written transposed (keys contiguous) for the attention kernel's P.V operand. Restates
//            kernels/glue/qkv_post.cc (q_post / k_post / v_post, lines 89-178) and redline/run_glue.py:27-37.
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace glue {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = float_to_bf16_bits(f[2 * i]) | (float_to_bf16_bits(f[2 * i + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// One warp per row; lane l owns the 8-value blocks kb = l, l + 32, ... of the row.
// params: bf16 [2][2][D] = {row 0: [g | sc], row 1: [g | sc]}; rows < row_split use row 1 (run_ln.py:82-86).
// The branch of a tensor-parallel row-split projection: the sum of the W ranks' bf16 partial outputs, each read from
// its rank's memory (this process's mapping of it; peers over NVLink), added in rank order in fp32 so that every
// rank forms the same value.
struct TpBranch {
  const uint16_t* const* parts;   // device array of W pointers, or null
  int W;
};
// Extra destinations of y (the tensor-parallel all-gather: this rank's rows of the LayerNorm output stored into every
// rank's copy of the next GEMM's A operand, peers over NVLink): a device array of n row-0 pointers, or n = 0.
struct YPeers {
  uint16_t* const* dst;
  int n;
};

__device__ __forceinline__ void load_branch(const void* br, int br_f32, TpBranch tp, int64_t r, int64_t D, int64_t kb,
                                            float (&f)[8]) {
  if (tp.W > 0) {
    // the partials are in the projection GEMM's chunk layout (rl_linear_bfp16_partial): 16-row x 32-column chunks of
    // 512 values, chunk (r / 16, column / 32); block kb (columns 8 kb .. 8 kb + 7) is 16 contiguous bytes of it
    const int64_t off = ((r >> 4) * (D >> 5) + (kb >> 2)) * 512 + (r & 15) * 32 + (kb & 3) * 8;
    unpack8(*reinterpret_cast<const uint4*>(tp.parts[0] + off), f);
    for (int w = 1; w < tp.W; ++w) {
      float g[8];
      unpack8(*reinterpret_cast<const uint4*>(tp.parts[w] + off), g);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] += g[i];
    }
  } else if (!br) {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = 0.0f;
  } else if (br_f32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(br) + r * D) + 2 * kb;
    const float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(br) + r * D) + kb), f);
  }
}

// The branch is bf16, or fp32 (the sum of tensor-parallel partial GEMM outputs), rounded to bf16 on load in both
// cases: x' = bf16(x + g * bf16(branch)).
// tp.W > 0: the branch is the TP sum (TpBranch); the kernel first waits until every other rank has signalled that its
// partial is complete (pad[r] >= epoch in this rank's signal pad, written by rl_tp_signal), a bounded wait that
// records kErrWaitTimeout and returns when it runs out.
__global__ void __launch_bounds__(kThreads) ln_mod_kernel(const uint16_t* __restrict__ x,
                                                          const void* __restrict__ br, int br_f32, TpBranch tp,
                                                          const unsigned long long* pad, int rank,
                                                          unsigned long long epoch,
                                                          const uint16_t* __restrict__ params, int64_t M, int64_t D,
                                                          int64_t row_split, float eps, int rms,
                                                          uint16_t* __restrict__ xo, uint16_t* __restrict__ y_dq,
                                                          uint8_t* __restrict__ y_q, YPeers yp) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t KB = D >> 3;
  if (tp.W > 0) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
      int ok = 1;
      for (int w = 0; ok && w < tp.W; ++w) {
        if (w == rank) continue;
        const long long t0 = clock64();
        while (true) {
          unsigned long long v;
          asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(pad + w) : "memory");
          if (v >= epoch) break;
          if (clock64() - t0 > RL_WAIT_LIMIT_CYCLES) {
            report(kErrWaitTimeout);
            ok = 0;
            break;
          }
          __nanosleep(200);
        }
      }
      ready = ok;
    }
    __syncthreads();
    if (!ready) return;
    br_f32 = 1;   // the fp32 sum is rounded to bf16 like an fp32 branch
  }
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + warp; r < M; r += static_cast<int64_t>(gridDim.x) * kWarps) {
    const uint16_t* prow = params + (r < row_split ? 2 * D : 0);
    const uint16_t* g = prow;
    const uint16_t* sc = prow + D;
    // pass 1: x' = bf16(x + g * branch) in float32 arithmetic (the products are exact: 8-bit x 8-bit significands)
    float s1 = 0.0f, s2 = 0.0f;
    for (int64_t kb = lane; kb < KB; kb += 32) {
      float xf[8], bf[8], gf[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(x + r * D) + kb), xf);
      unpack8(__ldg(reinterpret_cast<const uint4*>(g) + kb), gf);
      load_branch(br, br_f32, tp, r, D, kb, bf);
      if (br_f32) {
#pragma unroll
        for (int i = 0; i < 8; ++i) bf[i] = bf16_bits_to_float(float_to_bf16_bits(bf[i]));
      }
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] = bf16_bits_to_float(float_to_bf16_bits(__fadd_rn(xf[i], __fmul_rn(gf[i], bf[i]))));
        s1 += v[i];
        s2 = fmaf(v[i], v[i], s2);
      }
      if (xo) reinterpret_cast<uint4*>(xo + r * D)[kb] = pack8(v);
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    // LayerNorm, or RMSNorm (rms: no mean subtraction, the mean square as the variance)
    const float mean = rms ? 0.0f : s1 / static_cast<float>(D);
    const float var = rms ? s2 / static_cast<float>(D) : fmaxf(s2 / static_cast<float>(D) - mean * mean, 0.0f);
    const float rstd = 1.0f / sqrtf(var + eps);
    // pass 2: y = (x' - mean) * rstd * sc, rounded to bfp16 blocks of 8 along the row; x' is read back from xo
    // when the caller asked for it (each lane reads the blocks it wrote itself in pass 1)
    for (int64_t kb = lane; kb < KB; kb += 32) {
      float sf[8], v[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(sc) + kb), sf);
      if (xo) {
        unpack8(reinterpret_cast<const uint4*>(xo + r * D)[kb], v);
      } else {
        float xf[8], bf[8], gf[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(x + r * D) + kb), xf);
        unpack8(__ldg(reinterpret_cast<const uint4*>(g) + kb), gf);
        load_branch(br, br_f32, tp, r, D, kb, bf);
        if (br_f32) {
#pragma unroll
          for (int i = 0; i < 8; ++i) bf[i] = bf16_bits_to_float(float_to_bf16_bits(bf[i]));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = bf16_bits_to_float(float_to_bf16_bits(__fadd_rn(xf[i], __fmul_rn(gf[i], bf[i]))));
      }
      uint32_t bits[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) bits[i] = __float_as_uint((v[i] - mean) * rstd * sf[i]);
      uint32_t E, lo, hi, wq[4];
      bfp16_quant_block_fast(bits, E, lo, hi, wq);
      const uint4 yv = make_uint4(wq[0], wq[1], wq[2], wq[3]);
      if (y_dq) reinterpret_cast<uint4*>(y_dq + r * D)[kb] = yv;
      for (int i = 0; i < yp.n; ++i) reinterpret_cast<uint4*>(yp.dst[i] + r * D)[kb] = yv;
      if (y_q) {
        uint8_t* dst = y_q + (r * KB + kb) * 9;
        dst[0] = static_cast<uint8_t>(E);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dst[1 + i] = static_cast<uint8_t>(lo >> (8 * i));
          dst[5 + i] = static_cast<uint8_t>(hi >> (8 * i));
        }
      }
    }
  }
}

// The same math with one 128-thread CTA per row, for row counts too small to fill the GPU with one warp per row (the
// tensor-parallel row shards: 2176, 1088, 544 rows): thread t owns the blocks t, t + 128, ... (NB of them, D <=
// 8192), issues all of the row's loads before it uses any and keeps x' in registers between the passes, and the
// four warps add their sums once per row (in warp order: a fixed summation order). A warp-per-row pass walks the
// row's 12 blocks per lane one load at a time; with few rows that chain of dependent loads, not bandwidth, set the
// time (a LayerNorm of 1088 rows took as long as one of 4352).
constexpr int kRowThreads = 128;
constexpr int kRowMaxNB = 8;

template <int NB>
__global__ void __launch_bounds__(kRowThreads, NB <= 2 ? 8 : (NB <= 4 ? 6 : 4))
    ln_mod_row_kernel(const uint16_t* __restrict__ x, const void* __restrict__ br, int br_f32, TpBranch tp,
                      const unsigned long long* pad, int rank, unsigned long long epoch,
                      const uint16_t* __restrict__ params, int64_t M, int64_t D, int64_t row_split, float eps,
                      int rms, uint16_t* __restrict__ xo, uint16_t* __restrict__ y_dq, uint8_t* __restrict__ y_q,
                      YPeers yp) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int64_t KB = D >> 3;
  __shared__ float red[2][4][2];   // per-warp (sum, sum of squares), two rows apart
  if (tp.W > 0) {
    __shared__ int ready;
    if (t == 0) {
      int ok = 1;
      for (int w = 0; ok && w < tp.W; ++w) {
        if (w == rank) continue;
        const long long t0 = clock64();
        while (true) {
          unsigned long long v;
          asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(pad + w) : "memory");
          if (v >= epoch) break;
          if (clock64() - t0 > RL_WAIT_LIMIT_CYCLES) {
            report(kErrWaitTimeout);
            ok = 0;
            break;
          }
          __nanosleep(200);
        }
      }
      ready = ok;
    }
    __syncthreads();
    if (!ready) return;
    br_f32 = 1;
  }
  int it = 0;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x, ++it) {
    const uint16_t* prow = params + (r < row_split ? 2 * D : 0);
    uint4 xr[NB], gr[NB];
    float v[NB][8];
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int64_t kb = t + kRowThreads * i;
      if (kb < KB) {
        xr[i] = __ldg(reinterpret_cast<const uint4*>(x + r * D) + kb);
        gr[i] = __ldg(reinterpret_cast<const uint4*>(prow) + kb);
        load_branch(br, br_f32, tp, r, D, kb, v[i]);
      }
    }
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int64_t kb = t + kRowThreads * i;
      if (kb < KB) {
        float xf[8], gf[8];
        unpack8(xr[i], xf);
        unpack8(gr[i], gf);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float b = br_f32 ? bf16_bits_to_float(float_to_bf16_bits(v[i][j])) : v[i][j];
          v[i][j] = bf16_bits_to_float(float_to_bf16_bits(__fadd_rn(xf[j], __fmul_rn(gf[j], b))));
          s1 += v[i][j];
          s2 = fmaf(v[i][j], v[i][j], s2);
        }
        if (xo) reinterpret_cast<uint4*>(xo + r * D)[kb] = pack8(v[i]);
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) {
      red[it & 1][warp][0] = s1;
      red[it & 1][warp][1] = s2;
    }
    __syncthreads();   // a buffer is written again two rows later, after every thread passed the next row's barrier
    s1 = red[it & 1][0][0] + red[it & 1][1][0] + red[it & 1][2][0] + red[it & 1][3][0];
    s2 = red[it & 1][0][1] + red[it & 1][1][1] + red[it & 1][2][1] + red[it & 1][3][1];
    const float mean = rms ? 0.0f : s1 / static_cast<float>(D);
    const float var = rms ? s2 / static_cast<float>(D) : fmaxf(s2 / static_cast<float>(D) - mean * mean, 0.0f);
    const float rstd = 1.0f / sqrtf(var + eps);
    const uint16_t* sc = prow + D;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int64_t kb = t + kRowThreads * i;
      if (kb < KB) {
        float sf[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(sc) + kb), sf);
        uint32_t bits[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) bits[j] = __float_as_uint((v[i][j] - mean) * rstd * sf[j]);
        uint32_t E, lo, hi, wq[4];
        bfp16_quant_block_fast(bits, E, lo, hi, wq);
        const uint4 yv = make_uint4(wq[0], wq[1], wq[2], wq[3]);
        if (y_dq) reinterpret_cast<uint4*>(y_dq + r * D)[kb] = yv;
        for (int k = 0; k < yp.n; ++k) reinterpret_cast<uint4*>(yp.dst[k] + r * D)[kb] = yv;
        if (y_q) {
          uint8_t* dst = y_q + (r * KB + kb) * 9;
          dst[0] = static_cast<uint8_t>(E);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            dst[1 + j] = static_cast<uint8_t>(lo >> (8 * j));
            dst[5 + j] = static_cast<uint8_t>(hi >> (8 * j));
          }
        }
      }
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2_rn(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// One warp per token: lane l owns dims 4l..4l+3 (two RoPE pairs) of every q and k head; the token's (cos, sin) and
// the norm weights are loaded once.
__global__ void __launch_bounds__(kThreads) qk_norm_rope_tok_kernel(const uint16_t* __restrict__ qkv,
                                                                    const float* __restrict__ cs,
                                                                    const float* __restrict__ wq,
                                                                    const float* __restrict__ wk, int64_t M, int H,
                                                                    int Hkv, float eps, uint16_t* __restrict__ q,
                                                                    uint16_t* __restrict__ k) {
  // one warp per token; a half-warp per head (lane & 15 = 16-byte chunk of 8 dims = 4 RoPE pairs), so each step
  // covers two heads with fully coalesced 256-byte loads and a 16-lane (4-level) sum of squares
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hh = lane >> 4, c = lane & 15;
  const int64_t ld = static_cast<int64_t>(H + 2 * Hkv) * 128;   // [q H heads | k Hkv heads | v Hkv heads]
  const int nh = H + Hkv;                                           // normalised heads per token
  const float4 wq0 = __ldg(reinterpret_cast<const float4*>(wq) + 2 * c), wq1 = __ldg(reinterpret_cast<const float4*>(wq) + 2 * c + 1);
  const float4 wk0 = __ldg(reinterpret_cast<const float4*>(wk) + 2 * c), wk1 = __ldg(reinterpret_cast<const float4*>(wk) + 2 * c + 1);
  for (int64_t m = static_cast<int64_t>(blockIdx.x) * kWarps + warp; m < M; m += static_cast<int64_t>(gridDim.x) * kWarps) {
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(cs + m * 128) + 2 * c);      // (cos, sin) of pairs 4c, 4c+1
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(cs + m * 128) + 2 * c + 1);  // pairs 4c+2, 4c+3
    const uint16_t* row = qkv + m * ld;
#pragma unroll 4
    for (int i = 0; i < (nh + 1) / 2; ++i) {          // heads u = 2i + hh: u < H is q head u, else k head u - H
      const int u0 = 2 * i + hh;
      const bool valid = u0 < nh;                     // an odd head count leaves the last half-warp idle
      const int u = valid ? u0 : nh - 1;
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row + static_cast<int64_t>(u) * 128) + c);
      float v[8];
      const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = __uint_as_float(rw[j] << 16);
        v[2 * j + 1] = __uint_as_float(rw[j] & 0xFFFF0000u);
      }
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = 1.0f / sqrtf(ss * (1.0f / 128.0f) + eps);
      const bool isq = u < H;
      const float w[8] = {isq ? wq0.x : wk0.x, isq ? wq0.y : wk0.y, isq ? wq0.z : wk0.z, isq ? wq0.w : wk0.w,
                          isq ? wq1.x : wk1.x, isq ? wq1.y : wk1.y, isq ? wq1.z : wk1.z, isq ? wq1.w : wk1.w};
      const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      uint32_t out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float n0 = v[2 * j] * inv * w[2 * j], n1 = v[2 * j + 1] * inv * w[2 * j + 1];
        const float co = cc[2 * j], si = cc[2 * j + 1];
        out[j] = pack_bf16x2_rn(n0 * co - n1 * si, n0 * si + n1 * co);
      }
      uint16_t* dst = isq ? q + (static_cast<int64_t>(u) * M + m) * 128 : k + (static_cast<int64_t>(u - H) * M + m) * 128;
      if (valid) reinterpret_cast<uint4*>(dst)[c] = make_uint4(out[0], out[1], out[2], out[3]);
    }
  }
}

// V (token-major, 128 dims per head) -> V^T (head, dim, token), 64 tokens x 128 dims per CTA through shared memory.
// The tile is [128 dims][64 tokens] of bf16 with the 16-byte chunk index of a row XOR-ed with (dim / 8) & 7, so the
// transposing 2-byte stores (16 dim groups per warp) spread over 8 bank groups and the row reads stay 16-byte
// vectors.
__global__ void __launch_bounds__(kThreads) v_transpose16_kernel(const uint16_t* __restrict__ qkv, int64_t M, int H,
                                                                 int Hkv, int64_t ldv, uint16_t* __restrict__ vt) {
  __shared__ __align__(16) uint16_t tile[128 * 64];
  const int64_t ld = static_cast<int64_t>(H + 2 * Hkv) * 128;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int h = blockIdx.y;
  auto at = [](int d, int t) { return d * 64 + ((((t >> 3) ^ (d >> 3)) & 7) << 3) + (t & 7); };
#pragma unroll
  for (int it = 0; it < 4; ++it) {                    // 64 tokens x 16 chunks of 8 dims
    const int cid = threadIdx.x + it * kThreads;
    const int t = cid >> 4, dg = cid & 15;
    const int64_t m = m0 + t;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < M) v = __ldg(reinterpret_cast<const uint4*>(qkv + m * ld + (static_cast<int64_t>(H) + Hkv + h) * 128) + dg);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tile[at(8 * dg + 2 * i, t)] = static_cast<uint16_t>(wv[i]);
      tile[at(8 * dg + 2 * i + 1, t)] = static_cast<uint16_t>(wv[i] >> 16);
    }
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < 4; ++it) {                    // 128 dims x 8 chunks of 8 tokens
    const int cid = threadIdx.x + it * kThreads;
    const int d = cid >> 3, tc = cid & 7;
    const int64_t m = m0 + 8 * tc;
    if (m < ldv)
      *reinterpret_cast<uint4*>(vt + (static_cast<int64_t>(h) * 128 + d) * ldv + m) =
          *reinterpret_cast<const uint4*>(&tile[at(d, 8 * tc)]);
  }
}

inline int grid_rows(int64_t units, int per_cta) {
  const int64_t need = (units + per_cta - 1) / per_cta;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

// Residual + LayerNorm / RMSNorm launch (rl_ln_mod, rl_rms_mod, rl_ln_mod_tp, rl_ln_mod_tp_rs): one warp per row
// when there are rows for at least two warps per SM-slot of the grid (4352 rows of config 4), else one CTA per row
// (D <= 8192).
inline int launch_ln_mod(const uint16_t* x, const void* br, int br_f32, TpBranch tp, const unsigned long long* pad,
                         int rank, unsigned long long epoch, const uint16_t* params, int64_t M, int64_t D,
                         int64_t row_split, float eps, int rms, uint16_t* xo, uint16_t* y_dq, uint8_t* y_q,
                         cudaStream_t stream, YPeers yp = YPeers{nullptr, 0}) {
  const int nb = static_cast<int>(((D >> 3) + kRowThreads - 1) / kRowThreads);
  if (nb > kRowMaxNB || M > static_cast<int64_t>(sm_count()) * 2 * kWarps) {
    ln_mod_kernel<<<grid_rows(M, kWarps), kThreads, 0, stream>>>(x, br, br_f32, tp, pad, rank, epoch, params, M, D,
                                                                 row_split, eps, rms, xo, y_dq, y_q, yp);
  } else {
    const unsigned grid = static_cast<unsigned>(M);
#define RL_LN_ROW(N)                                                                                                \
  case N:                                                                                                           \
    ln_mod_row_kernel<N><<<grid, kRowThreads, 0, stream>>>(x, br, br_f32, tp, pad, rank, epoch, params, M, D,      \
                                                           row_split, eps, rms, xo, y_dq, y_q, yp);                 \
    break;
    switch (nb) {
      RL_LN_ROW(1) RL_LN_ROW(2) RL_LN_ROW(3) RL_LN_ROW(4) RL_LN_ROW(5) RL_LN_ROW(6) RL_LN_ROW(7) RL_LN_ROW(8)
      default: break;
    }
#undef RL_LN_ROW
  }
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

}  // namespace glue
}  // namespace rl

namespace rl {
static int norm_mod(const char* fn, int rms, const uint16_t* x, const void* branch, int branch_dtype, const uint16_t* params, int64_t M, int64_t D,
                    int64_t row_split, uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream) {
  RL_REQUIRE(x && params, RL_ERR_ARGUMENT, "%s: NULL pointer", fn);
  RL_REQUIRE(M >= 0 && D >= 8 && D % 8 == 0, RL_ERR_ARGUMENT, "%s: need D %% 8 == 0", fn);
  RL_REQUIRE(branch_dtype == RL_BF16 || branch_dtype == RL_F32, RL_ERR_ARGUMENT, "%s: bad branch dtype", fn);
  RL_REQUIRE(aligned(x, 16) && aligned(branch, 16) && aligned(params, 16) && aligned(x_out, 16) && aligned(y_dq, 16),
             RL_ERR_ALIGNMENT, "%s: bf16 pointers must be 16-byte aligned", fn);
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "%s: needs an sm_100 device", fn);
  if (M == 0) return RL_OK;
  return glue::launch_ln_mod(x, branch, branch_dtype == RL_F32 ? 1 : 0, glue::TpBranch{nullptr, 0}, nullptr, 0, 0ull,
                             params, M, D, row_split, 1e-6f, rms, x_out, y_dq, y_q, stream);
}
}  // namespace rl

extern "C" {

int rl_ln_mod(const uint16_t* x, const void* branch, int branch_dtype, const uint16_t* params, int64_t M, int64_t D,
              int64_t row_split, uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream) {
  return rl::norm_mod("rl_ln_mod", 0, x, branch, branch_dtype, params, M, D, row_split, x_out, y_dq, y_q, stream);
}

int rl_rms_mod(const uint16_t* x, const void* branch, int branch_dtype, const uint16_t* params, int64_t M, int64_t D,
               int64_t row_split, uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream) {
  return rl::norm_mod("rl_rms_mod", 1, x, branch, branch_dtype, params, M, D, row_split, x_out, y_dq, y_q, stream);
}

int rl_qkv_post_gqa(const uint16_t* qkv, const float* rope_cs, const float* w_q, const float* w_k, int64_t M, int H,
                    int Hkv, uint16_t* q, uint16_t* k, uint16_t* vt, int64_t ldv, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(qkv && rope_cs && w_q && w_k && q && k && vt, RL_ERR_ARGUMENT, "rl_qkv_post: NULL pointer");
  RL_REQUIRE(M >= 0 && H > 0 && Hkv > 0 && ldv >= M && ldv % 8 == 0, RL_ERR_ARGUMENT,
             "rl_qkv_post: need ldv >= M and ldv %% 8 == 0");
  RL_REQUIRE(aligned(qkv, 16) && aligned(rope_cs, 16) && aligned(w_q, 16) && aligned(w_k, 16) && aligned(q, 16) &&
                 aligned(k, 16) && aligned(vt, 16),
             RL_ERR_ALIGNMENT, "rl_qkv_post: pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_qkv_post: needs an sm_100 device");
  if (M == 0) return RL_OK;
  glue::qk_norm_rope_tok_kernel<<<glue::grid_rows(M, glue::kWarps), glue::kThreads, 0, stream>>>(
      qkv, rope_cs, w_q, w_k, M, H, Hkv, 1e-6f, q, k);
  RL_TRY_CUDA(cudaGetLastError());
  const dim3 grid(static_cast<unsigned>((ldv + 63) / 64), static_cast<unsigned>(Hkv));
  glue::v_transpose16_kernel<<<grid, glue::kThreads, 0, stream>>>(qkv, M, H, Hkv, ldv, vt);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_qkv_post(const uint16_t* qkv, const float* rope_cs, const float* w_q, const float* w_k, int64_t M, int H,
                uint16_t* q, uint16_t* k, uint16_t* vt, int64_t ldv, rl_stream_t stream) {
  return rl_qkv_post_gqa(qkv, rope_cs, w_q, w_k, M, H, H, q, k, vt, ldv, stream);
}

}  // extern "C"
