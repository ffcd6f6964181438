// bfp16 codec kernels: activation quantiser / decoder, the reference's packed-weight stream, and the GPU-native
// weight tile format the GEMM consumes. All are HBM-bound byte work: one thread owns one 8-value block, loads it
// with 128-bit vector loads, and a warp writes its 32 x 9 = 288 output bytes as 18 aligned 16-byte stores through
// a shared-memory staging line.
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace codec {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStageBytes = 32 * 9;  // one warp's blocks

// Source coordinates (row, first column) of output block `ob` of an (M, K) matrix in the given stream order.
//   RL_ROWMAJOR : block (r, c/8) at r*K/8 + c/8;
//   RL_A_LAYOUT : a_layout(., 128, 64) (npu_layouts.py:18-23): 1024 blocks per tile; inside (sbr, bc, bis, rib);
//   RL_C_ATB    : c_layout_atb(., 128, 128) (npu_layouts.py:31-48): groups of 4 x 8 tiles of 128 x 128, per group
//                 one chunk per core column stacking its 4 row tiles; inside 2x2 super-blocks of row-major 8x8.
__device__ __forceinline__ void block_coords(int layout, int64_t ob, int64_t K, int64_t& r, int64_t& c0) {
  if (layout == RL_ROWMAJOR) {
    const int64_t kb = K >> 3;
    r = ob / kb;
    c0 = (ob - r * kb) << 3;
  } else if (layout == RL_A_LAYOUT) {
    const int64_t tile = ob >> 10;
    const int w = static_cast<int>(ob & 1023);
    const int64_t kt_n = K >> 6;
    const int64_t tr = tile / kt_n, tc = tile - tr * kt_n;
    const int sbr = w >> 7, bc = (w >> 4) & 7, bis = (w >> 3) & 1, rib = w & 7;
    r = tr * 128 + sbr * 16 + bis * 8 + rib;
    c0 = tc * 64 + bc * 8;
  } else {  // RL_C_ATB: ob = ((((((rg*CG + cg)*8 + col)*4 + row)*8 + sbr)*8 + sbc)*2 + br)*2 + bc)*8 + rib
    int64_t t = ob;
    const int rib = static_cast<int>(t & 7); t >>= 3;
    const int bc = static_cast<int>(t & 1); t >>= 1;
    const int br = static_cast<int>(t & 1); t >>= 1;
    const int sbc = static_cast<int>(t & 7); t >>= 3;
    const int sbr = static_cast<int>(t & 7); t >>= 3;
    const int row = static_cast<int>(t & 3); t >>= 2;
    const int col = static_cast<int>(t & 7); t >>= 3;
    const int64_t cgn = K >> 10;
    const int64_t rg = t / cgn, cg = t - rg * cgn;
    r = rg * 512 + row * 128 + sbr * 16 + br * 8 + rib;
    c0 = cg * 1024 + col * 128 + sbc * 16 + bc * 8;
  }
}

// Inverse of block_coords: the stream block index of the 8 values (r, c0 .. c0+7).
__device__ __forceinline__ int64_t block_index(int layout, int64_t r, int64_t c0, int64_t K) {
  if (layout == RL_ROWMAJOR) return r * (K >> 3) + (c0 >> 3);
  if (layout == RL_A_LAYOUT) {
    const int64_t tile = (r >> 7) * (K >> 6) + (c0 >> 6);
    const int64_t w = ((((r & 127) >> 4) * 8 + ((c0 & 63) >> 3)) * 2 + ((r >> 3) & 1)) * 8 + (r & 7);
    return tile * 1024 + w;
  }
  const int64_t rg = r >> 9, row = (r >> 7) & 3, sbr = (r >> 4) & 7, br = (r >> 3) & 1, rib = r & 7;
  const int64_t cg = c0 >> 10, col = (c0 >> 7) & 7, sbc = (c0 >> 4) & 7, bc = (c0 >> 3) & 1;
  int64_t i = (rg * (K >> 10) + cg) * 8 + col;
  i = ((((i * 4 + row) * 8 + sbr) * 8 + sbc) * 2 + br) * 2 + bc;
  return i * 8 + rib;
}

inline bool layout_ok(int layout, int64_t M, int64_t K) {
  if (layout == RL_ROWMAJOR) return K % 8 == 0;
  if (layout == RL_A_LAYOUT) return M % 128 == 0 && K % 64 == 0;
  if (layout == RL_C_ATB) return M % 512 == 0 && K % 1024 == 0;
  return false;
}

template <typename T>
__device__ __forceinline__ void load_block(const T* __restrict__ p, uint32_t (&b)[8]);

template <>
__device__ __forceinline__ void load_block<float>(const float* __restrict__ p, uint32_t (&b)[8]) {
  const uint4 v0 = __ldg(reinterpret_cast<const uint4*>(p));
  const uint4 v1 = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  b[0] = v0.x; b[1] = v0.y; b[2] = v0.z; b[3] = v0.w;
  b[4] = v1.x; b[5] = v1.y; b[6] = v1.z; b[7] = v1.w;
}

template <>
__device__ __forceinline__ void load_block<uint16_t>(const uint16_t* __restrict__ p, uint32_t (&b)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    b[2 * i] = w[i] << 16;
    b[2 * i + 1] = w[i] & 0xFFFF0000u;
  }
}

// Quantise one block: exponent byte E and the 8 mantissas packed as bytes into (lo, hi).
__device__ __forceinline__ void quant_block(const uint32_t (&b)[8], uint32_t& E, uint32_t& lo, uint32_t& hi) {
  E = bfp16_block_exponent(b);
  lo = hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo |= (static_cast<uint32_t>(bfp16_quant_one(b[i], E)) & 0xFFu) << (8 * i);
    hi |= (static_cast<uint32_t>(bfp16_quant_one(b[4 + i], E)) & 0xFFu) << (8 * i);
  }
}

__device__ __forceinline__ void stage_put(uint8_t* st, int lane, uint32_t E, uint32_t lo, uint32_t hi) {
  uint8_t* p = st + lane * 9;
  p[0] = static_cast<uint8_t>(E);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    p[1 + i] = static_cast<uint8_t>(lo >> (8 * i));
    p[5 + i] = static_cast<uint8_t>(hi >> (8 * i));
  }
}

__device__ __forceinline__ void stage_get(const uint8_t* st, int lane, uint32_t& E, uint32_t& lo, uint32_t& hi) {
  const uint8_t* p = st + lane * 9;
  E = p[0];
  lo = hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo |= static_cast<uint32_t>(p[1 + i]) << (8 * i);
    hi |= static_cast<uint32_t>(p[5 + i]) << (8 * i);
  }
}

// Write a warp's staged blocks [base, base + 32) to dst (16-byte aligned stream of 9-byte blocks).
__device__ __forceinline__ void stage_flush(const uint8_t* st, uint8_t* __restrict__ dst, int64_t base,
                                            int64_t nblocks, int lane) {
  __syncwarp();
  if (base + 32 <= nblocks) {
    if (lane < 18)
      reinterpret_cast<uint4*>(dst + base * 9)[lane] = reinterpret_cast<const uint4*>(st)[lane];
  } else {
    const int nbytes = static_cast<int>(nblocks - base) * 9;
    for (int i = lane; i < nbytes; i += 32) dst[base * 9 + i] = st[i];
  }
  __syncwarp();
}

// Load a warp's 32 source blocks [base, base + 32) into the staging line.
__device__ __forceinline__ void stage_fill(uint8_t* st, const uint8_t* __restrict__ src, int64_t base,
                                           int64_t nblocks, int lane) {
  __syncwarp();
  if (base + 32 <= nblocks) {
    if (lane < 18) reinterpret_cast<uint4*>(st)[lane] = __ldg(reinterpret_cast<const uint4*>(src + base * 9) + lane);
  } else {
    const int nbytes = static_cast<int>(nblocks - base) * 9;
    for (int i = lane; i < nbytes; i += 32) st[i] = src[base * 9 + i];
  }
  __syncwarp();
}

template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_kernel(const T* __restrict__ x, int64_t K, int layout,
                                                            uint8_t* __restrict__ q, uint16_t* __restrict__ dq,
                                                            int64_t nblocks) {
  __shared__ __align__(16) uint8_t stage[kWarps][kStageBytes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads + warp * 32; base < nblocks; base += stride) {
    const int64_t ob = base + lane;
    if (ob < nblocks) {
      // row-major blocks are contiguous: block ob starts at value 8 * ob, no division needed
      int64_t off = ob * 8;
      if (layout != RL_ROWMAJOR) {
        int64_t r, c0;
        block_coords(layout, ob, K, r, c0);
        off = r * K + c0;
      }
      uint32_t b[8];
      load_block<T>(x + off, b);
      uint32_t E, lo, hi, w[4];
      bfp16_quant_block_fast(b, E, lo, hi, w);
      if (dq) *reinterpret_cast<uint4*>(dq + off) = make_uint4(w[0], w[1], w[2], w[3]);
      if (q) stage_put(stage[warp], lane, E, lo, hi);
    }
    if (q) stage_flush(stage[warp], q, base, nblocks, lane);
  }
}

// The GEMM's A operand alone (row-major blocks, decoded values only, no bytes): each thread quantises kUnroll blocks
// per pass, their loads issued together (kUnroll x 16 or 32 bytes in flight per thread instead of one block's), the
// blocks of a pass kThreads apart so every load and store of a warp stays one contiguous 512-byte run.
constexpr int kUnroll = 4;
template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_dq_kernel(const T* __restrict__ x, uint16_t* __restrict__ dq,
                                                               int64_t nblocks) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads * kUnroll;
  for (int64_t b0 = static_cast<int64_t>(blockIdx.x) * kThreads * kUnroll + threadIdx.x; b0 < nblocks; b0 += step) {
    uint32_t b[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t ob = b0 + static_cast<int64_t>(u) * kThreads;
      if (ob < nblocks) load_block<T>(x + ob * 8, b[u]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t ob = b0 + static_cast<int64_t>(u) * kThreads;
      if (ob < nblocks) {
        uint32_t E, lo, hi, w[4];
        bfp16_quant_block_fast(b[u], E, lo, hi, w);
        *reinterpret_cast<uint4*>(dq + ob * 8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// bf16 (M, K) in one stream order -> another; the orders keep 8 consecutive columns together, so 16-byte moves.
__global__ void __launch_bounds__(kThreads) permute_bf16_kernel(const uint16_t* __restrict__ src, int src_layout,
                                                                uint16_t* __restrict__ dst, int dst_layout, int64_t K,
                                                                int64_t nblocks) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t ob = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; ob < nblocks; ob += stride) {
    int64_t r, c0;
    block_coords(dst_layout, ob, K, r, c0);
    const int64_t ib = block_index(src_layout, r, c0, K);
    reinterpret_cast<uint4*>(dst)[ob] = __ldg(reinterpret_cast<const uint4*>(src) + ib);
  }
}

template <typename TO>
__global__ void __launch_bounds__(kThreads) dequantize_kernel(const uint8_t* __restrict__ q, int64_t K, int layout,
                                                              TO* __restrict__ out, int64_t nblocks) {
  __shared__ __align__(16) uint8_t stage[kWarps][kStageBytes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads + warp * 32; base < nblocks; base += stride) {
    stage_fill(stage[warp], q, base, nblocks, lane);
    const int64_t ob = base + lane;
    if (ob < nblocks) {
      uint32_t E, lo, hi;
      stage_get(stage[warp], lane, E, lo, hi);
      uint32_t w[4];
      bfp16_decode_block(E, lo, hi, w);
      int64_t r, c0;
      block_coords(layout, ob, K, r, c0);
      if constexpr (sizeof(TO) == 2) {
        *reinterpret_cast<uint4*>(out + r * K + c0) = make_uint4(w[0], w[1], w[2], w[3]);
      } else {
        uint4* o = reinterpret_cast<uint4*>(out + r * K + c0);
        o[0] = make_uint4(w[0] << 16, w[0] & 0xFFFF0000u, w[1] << 16, w[1] & 0xFFFF0000u);
        o[1] = make_uint4(w[2] << 16, w[2] & 0xFFFF0000u, w[3] << 16, w[3] & 0xFFFF0000u);
      }
    }
  }
}

// ---- weights ------------------------------------------------------------------------------------------------

// Block `ib` (0..1023) of a 64 x 128 b_layout tile: column n (0..127) and 8-row block bk (0..7).
__device__ __forceinline__ void b_tile_block(int ib, int& n, int& bk) {
  const int col = ib & 7, bis = (ib >> 3) & 1, bk_ = (ib >> 4) & 7, sbc = ib >> 7;
  n = sbc * 16 + bis * 8 + col;
  bk = bk_;
}

// Native row of tile column n: identity, or (swiglu) quarter q holds gate units 16q.. then proj units 16q..
__device__ __forceinline__ int native_row(int n, int swiglu) {
  if (!swiglu) return n;
  const int u = n & 63;
  return 32 * (u >> 4) + (n >= 64 ? 16 : 0) + (u & 15);
}

// Native tiles keep the mantissas in offset binary (m + 128), which saves the GEMM's decoder one XOR per word.
__device__ __forceinline__ void native_put(uint8_t* __restrict__ tile, int row, int bk, uint32_t E, uint32_t lo,
                                           uint32_t hi) {
  *reinterpret_cast<uint2*>(tile + ((bk >> 1) * 128 + row) * 16 + (bk & 1) * 8) =
      make_uint2(lo ^ 0x80808080u, hi ^ 0x80808080u);
  tile[8192 + row * 8 + bk] = static_cast<uint8_t>(E);
}

template <typename T>
__device__ __forceinline__ void load_column_block(const T* __restrict__ B, int64_t N, int64_t k0, int64_t n,
                                                  uint32_t (&b)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (sizeof(T) == 4)
      b[i] = __float_as_uint(__ldg(B + (k0 + i) * N + n));
    else
      b[i] = static_cast<uint32_t>(__ldg(B + (k0 + i) * N + n)) << 16;
  }
}

// Float B (K, N) -> the reference's stream to_bfp16(b_layout(B, 64, 128)) (pack_weights.py:72-79).
template <typename T>
__global__ void __launch_bounds__(kThreads) pack_b_kernel(const T* __restrict__ B, int64_t K, int64_t N,
                                                          uint8_t* __restrict__ out, int64_t nblocks) {
  __shared__ __align__(16) uint8_t stage[kWarps][kStageBytes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t KT = K >> 6;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads + warp * 32; base < nblocks; base += stride) {
    const int64_t ob = base + lane;
    if (ob < nblocks) {
      const int64_t tile = ob >> 10;
      const int64_t nt = tile / KT, kt = tile - nt * KT;
      int n, bk;
      b_tile_block(static_cast<int>(ob & 1023), n, bk);
      uint32_t b[8];
      load_column_block<T>(B, N, kt * 64 + bk * 8, nt * 128 + n, b);
      uint32_t E, lo, hi;
      quant_block(b, E, lo, hi);
      stage_put(stage[warp], lane, E, lo, hi);
    }
    stage_flush(stage[warp], out, base, nblocks, lane);
  }
}

// The reference stream -> native tiles (tile order unchanged; blocks regrouped inside each 9216-byte tile).
__global__ void __launch_bounds__(kThreads) native_from_pack_b_kernel(const uint8_t* __restrict__ packed,
                                                                      int swiglu, uint8_t* __restrict__ native,
                                                                      int64_t nblocks) {
  __shared__ __align__(16) uint8_t stage[kWarps][kStageBytes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads + warp * 32; base < nblocks; base += stride) {
    stage_fill(stage[warp], packed, base, nblocks, lane);
    const int64_t ob = base + lane;
    if (ob < nblocks) {
      uint32_t E, lo, hi;
      stage_get(stage[warp], lane, E, lo, hi);
      int n, bk;
      b_tile_block(static_cast<int>(ob & 1023), n, bk);
      native_put(native + (ob >> 10) * 9216, native_row(n, swiglu), bk, E, lo, hi);
    }
  }
}

// Float B (K, N) -> native tiles directly; one thread per (column, 8-row block), columns fastest for coalescing.
template <typename T>
__global__ void __launch_bounds__(kThreads) pack_native_kernel(const T* __restrict__ B, int64_t K, int64_t N,
                                                               int swiglu, uint8_t* __restrict__ native,
                                                               int64_t nblocks) {
  const int64_t KT = K >> 6;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t ob = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; ob < nblocks; ob += stride) {
    // ob = ((kb) * N + n): kb = global 8-row block index
    const int64_t kb = ob / N, n = ob - kb * N;
    uint32_t b[8];
    load_column_block<T>(B, N, kb * 8, n, b);
    uint32_t E, lo, hi;
    quant_block(b, E, lo, hi);
    const int64_t nt = n >> 7, kt = kb >> 3;
    native_put(native + (nt * KT + kt) * 9216, native_row(static_cast<int>(n & 127), swiglu),
               static_cast<int>(kb & 7), E, lo, hi);
  }
}

inline int grid_for(int64_t work, int threads = kThreads) {
  const int64_t need = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace codec
}  // namespace rl

using namespace rl;

extern "C" {

int rl_quantize_bfp16(const void* x, int x_dtype, int64_t M, int64_t K, int layout, uint8_t* q_out,
                      uint16_t* dq_out, rl_stream_t stream) {
  RL_REQUIRE(x != nullptr, RL_ERR_ARGUMENT, "rl_quantize_bfp16: x is NULL");
  RL_REQUIRE(M >= 0 && K > 0 && K % 8 == 0, RL_ERR_ARGUMENT, "rl_quantize_bfp16: need K %% 8 == 0 (M=%lld K=%lld)",
             (long long)M, (long long)K);
  RL_REQUIRE(x_dtype == RL_F32 || x_dtype == RL_BF16, RL_ERR_ARGUMENT, "rl_quantize_bfp16: bad dtype %d", x_dtype);
  RL_REQUIRE(layout == RL_ROWMAJOR || layout == RL_A_LAYOUT || layout == RL_C_ATB, RL_ERR_ARGUMENT,
             "rl_quantize_bfp16: bad layout %d", layout);
  RL_REQUIRE(codec::layout_ok(layout, M, K), RL_ERR_ARGUMENT,
             "rl_quantize_bfp16: layout %d needs M %% 128 and K %% 64 (a_layout) or M %% 512 and K %% 1024 (C order)",
             layout);
  RL_REQUIRE(aligned(x, 16) && aligned(q_out, 16) && aligned(dq_out, 16), RL_ERR_ALIGNMENT,
             "rl_quantize_bfp16: pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_quantize_bfp16: needs an sm_100 device");
  const int64_t nblocks = M * K / 8;
  if (nblocks == 0) return RL_OK;
  if (!q_out && dq_out && layout == RL_ROWMAJOR) {   // decoded values only (the GEMM's A operand): the unrolled kernel
    // as many CTAs as are resident at once (one wave; the threads stride over the rest): a grid of several partial
    // waves left the last one mostly idle (11.7 us for config 1's X against 8.2 us of HBM time)
    const int per_pass = codec::kThreads * codec::kUnroll;
    const int64_t need = (nblocks + per_pass - 1) / per_pass;
    int resident = 0;
    if (x_dtype == RL_F32) {
      RL_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, codec::quantize_dq_kernel<float>,
                                                                codec::kThreads, 0));
    } else {
      RL_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, codec::quantize_dq_kernel<uint16_t>,
                                                                codec::kThreads, 0));
    }
    const int64_t wave = static_cast<int64_t>(resident > 0 ? resident : 1) * sm_count();
    const int g = static_cast<int>(need < wave ? need : wave);
    if (x_dtype == RL_F32)
      codec::quantize_dq_kernel<float><<<g, codec::kThreads, 0, stream>>>(static_cast<const float*>(x), dq_out,
                                                                          nblocks);
    else
      codec::quantize_dq_kernel<uint16_t><<<g, codec::kThreads, 0, stream>>>(static_cast<const uint16_t*>(x),
                                                                             dq_out, nblocks);
    RL_TRY_CUDA(cudaGetLastError());
    return RL_OK;
  }
  const int grid = codec::grid_for(nblocks);
  if (x_dtype == RL_F32)
    codec::quantize_kernel<float><<<grid, codec::kThreads, 0, stream>>>(static_cast<const float*>(x), K, layout,
                                                                        q_out, dq_out, nblocks);
  else
    codec::quantize_kernel<uint16_t><<<grid, codec::kThreads, 0, stream>>>(static_cast<const uint16_t*>(x), K,
                                                                           layout, q_out, dq_out, nblocks);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_dequantize_bfp16(const uint8_t* q, int layout, int64_t M, int64_t K, void* out, int out_dtype,
                        rl_stream_t stream) {
  RL_REQUIRE(q != nullptr && out != nullptr, RL_ERR_ARGUMENT, "rl_dequantize_bfp16: NULL pointer");
  RL_REQUIRE(M >= 0 && K > 0 && K % 8 == 0, RL_ERR_ARGUMENT, "rl_dequantize_bfp16: need K %% 8 == 0");
  RL_REQUIRE(out_dtype == RL_F32 || out_dtype == RL_BF16, RL_ERR_ARGUMENT, "rl_dequantize_bfp16: bad dtype");
  RL_REQUIRE((layout == RL_ROWMAJOR || layout == RL_A_LAYOUT || layout == RL_C_ATB) &&
                 codec::layout_ok(layout, M, K),
             RL_ERR_ARGUMENT, "rl_dequantize_bfp16: bad layout / shape");
  RL_REQUIRE(aligned(q, 16) && aligned(out, 16), RL_ERR_ALIGNMENT, "rl_dequantize_bfp16: pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_dequantize_bfp16: needs an sm_100 device");
  const int64_t nblocks = M * K / 8;
  if (nblocks == 0) return RL_OK;
  const int grid = codec::grid_for(nblocks);
  if (out_dtype == RL_F32)
    codec::dequantize_kernel<float><<<grid, codec::kThreads, 0, stream>>>(q, K, layout, static_cast<float*>(out),
                                                                          nblocks);
  else
    codec::dequantize_kernel<uint16_t><<<grid, codec::kThreads, 0, stream>>>(q, K, layout,
                                                                             static_cast<uint16_t*>(out), nblocks);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_permute_bf16(const uint16_t* src, int src_layout, uint16_t* dst, int dst_layout, int64_t M, int64_t K,
                    rl_stream_t stream) {
  RL_REQUIRE(src && dst && src != dst, RL_ERR_ARGUMENT, "rl_permute_bf16: NULL or aliased pointers");
  RL_REQUIRE(src_layout >= RL_ROWMAJOR && src_layout <= RL_C_ATB && dst_layout >= RL_ROWMAJOR &&
                 dst_layout <= RL_C_ATB && codec::layout_ok(src_layout, M, K) && codec::layout_ok(dst_layout, M, K),
             RL_ERR_ARGUMENT, "rl_permute_bf16: bad layout / shape");
  RL_REQUIRE(aligned(src, 16) && aligned(dst, 16), RL_ERR_ALIGNMENT, "rl_permute_bf16: pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_permute_bf16: needs an sm_100 device");
  const int64_t nblocks = M * K / 8;
  if (nblocks == 0) return RL_OK;
  codec::permute_bf16_kernel<<<codec::grid_for(nblocks), codec::kThreads, 0, stream>>>(src, src_layout, dst,
                                                                                         dst_layout, K, nblocks);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_pack_b(const void* B, int dtype, int64_t K, int64_t N, uint8_t* out, rl_stream_t stream) {
  RL_REQUIRE(B != nullptr && out != nullptr, RL_ERR_ARGUMENT, "rl_pack_b: NULL pointer");
  RL_REQUIRE(K > 0 && N > 0 && K % 64 == 0 && N % 128 == 0, RL_ERR_ARGUMENT,
             "rl_pack_b: need K %% 64 == 0 and N %% 128 == 0 (K=%lld N=%lld)", (long long)K, (long long)N);
  RL_REQUIRE(dtype == RL_F32 || dtype == RL_BF16, RL_ERR_ARGUMENT, "rl_pack_b: bad dtype");
  RL_REQUIRE(aligned(out, 16), RL_ERR_ALIGNMENT, "rl_pack_b: out must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_pack_b: needs an sm_100 device");
  const int64_t nblocks = K * N / 8;
  const int grid = codec::grid_for(nblocks);
  if (dtype == RL_F32)
    codec::pack_b_kernel<float><<<grid, codec::kThreads, 0, stream>>>(static_cast<const float*>(B), K, N, out,
                                                                      nblocks);
  else
    codec::pack_b_kernel<uint16_t><<<grid, codec::kThreads, 0, stream>>>(static_cast<const uint16_t*>(B), K, N,
                                                                         out, nblocks);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_weights_from_pack_b(const uint8_t* packed, int64_t K, int64_t N, int swiglu_interleaved, uint8_t* native,
                           rl_stream_t stream) {
  RL_REQUIRE(packed != nullptr && native != nullptr, RL_ERR_ARGUMENT, "rl_weights_from_pack_b: NULL pointer");
  RL_REQUIRE(K > 0 && N > 0 && K % 64 == 0 && N % 128 == 0, RL_ERR_ARGUMENT,
             "rl_weights_from_pack_b: need K %% 64 == 0 and N %% 128 == 0");
  RL_REQUIRE(aligned(packed, 16) && aligned(native, 16), RL_ERR_ALIGNMENT,
             "rl_weights_from_pack_b: pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_weights_from_pack_b: needs an sm_100 device");
  const int64_t nblocks = K * N / 8;
  codec::native_from_pack_b_kernel<<<codec::grid_for(nblocks), codec::kThreads, 0, stream>>>(
      packed, swiglu_interleaved ? 1 : 0, native, nblocks);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_pack_weights(const void* B, int dtype, int64_t K, int64_t N, int swiglu_interleaved, uint8_t* native,
                    rl_stream_t stream) {
  RL_REQUIRE(B != nullptr && native != nullptr, RL_ERR_ARGUMENT, "rl_pack_weights: NULL pointer");
  RL_REQUIRE(K > 0 && N > 0 && K % 64 == 0 && N % 128 == 0, RL_ERR_ARGUMENT,
             "rl_pack_weights: need K %% 64 == 0 and N %% 128 == 0");
  RL_REQUIRE(dtype == RL_F32 || dtype == RL_BF16, RL_ERR_ARGUMENT, "rl_pack_weights: bad dtype");
  RL_REQUIRE(aligned(native, 16), RL_ERR_ALIGNMENT, "rl_pack_weights: native must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_pack_weights: needs an sm_100 device");
  const int64_t nblocks = K * N / 8;
  const int grid = codec::grid_for(nblocks);
  if (dtype == RL_F32)
    codec::pack_native_kernel<float><<<grid, codec::kThreads, 0, stream>>>(static_cast<const float*>(B), K, N,
                                                                           swiglu_interleaved ? 1 : 0, native,
                                                                           nblocks);
  else
    codec::pack_native_kernel<uint16_t><<<grid, codec::kThreads, 0, stream>>>(static_cast<const uint16_t*>(B), K,
                                                                              N, swiglu_interleaved ? 1 : 0,
                                                                              native, nblocks);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_weights_shard(int64_t K, int64_t N, int rank, int world, int64_t* n0, int64_t* n_cols, int64_t* byte_offset,
                     int64_t* byte_count) {
  RL_REQUIRE(n0 && n_cols && byte_offset && byte_count, RL_ERR_ARGUMENT, "rl_weights_shard: NULL pointer");
  RL_REQUIRE(world > 0 && rank >= 0 && rank < world, RL_ERR_ARGUMENT, "rl_weights_shard: rank %d of %d", rank, world);
  RL_REQUIRE(K > 0 && K % 64 == 0 && N > 0 && N % (128 * static_cast<int64_t>(world)) == 0, RL_ERR_ARGUMENT,
             "rl_weights_shard: need K %% 64 == 0 and N %% (128 * world) == 0 (K=%lld N=%lld world=%d)", (long long)K,
             (long long)N, world);
  // one 128-column strip = K / 64 tiles of 9216 bytes, contiguous in both the b_layout stream and the native format
  const int64_t cols = N / world, strip = K / 64 * 9216;
  *n0 = rank * cols;
  *n_cols = cols;
  *byte_offset = (rank * cols / 128) * strip;
  *byte_count = cols / 128 * strip;
  return RL_OK;
}

}  // extern "C"
