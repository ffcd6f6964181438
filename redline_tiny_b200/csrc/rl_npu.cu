// The NPU attention formats, for the drop-in of the reference's QKV-post and attention artifacts.
//
// The reference's QKV-post kernel (kernels/glue/qkv_post.cc; host side redline/run_qkv.py:41-79) writes, per head h
// and 64-token tile t, bfp16 streams that its attention kernels (kernels/attn/attn_bfp.cc; run_attn.py:29-35,
// 82-92) read:
//   Q[h][t]       = to_bfp16(a_layout(Q_h[64t .. 64t + 63], 64, 128))            (npu_layouts.py:18-23)
//   KV[h][t][0]   = to_bfp16(b_layout(K_h[64t .. 64t + 63]^T, 128, 64))          (npu_layouts.py:11-16)
//   KV[h][t][1]   = to_bfp16(b_layout(V_h[64t .. 64t + 63], 64, 128))
// each tile 1024 blocks of 9 bytes. Every block holds 8 values that are contiguous in this library's attention
// operands - q (H, rows, 128) and k (H, keys, 128) along the head dim, vt (H, 128, ldv) along the keys - so one thread
// per block converts between the two without staging. The per-block RoPE / norm table of the QKV-post kernel
// (run_qkv.qkv_tables, run_qkv.py:60-72) is decoded into the row-major (cos, sin) table and the two norm weights.
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace npu {

constexpr int kTileBlocks = 64 * 128 / 8;       // 1024 blocks per 64 x 128 tile
constexpr int kTileBytes = kTileBlocks * 9;     // 9216
constexpr int kTabRow = 128 * 64 + 2 * 128;     // 8448 bf16 per 64-row tile of the QKV table
constexpr int kThreads = 256;

// Block b (0 .. 1023) of a Q tile: a_layout(x, 64, 128) -> (row in tile, 8-dim group).
__device__ __forceinline__ void q_block(int b, int& row, int& dg) {
  const int rib = b & 7, bis = (b >> 3) & 1, bc = (b >> 4) & 15, sbr = b >> 8;
  row = sbr * 16 + bis * 8 + rib;
  dg = bc;
}
// Block b of a K tile: b_layout(K_t^T, 128, 64) -> (key in tile, 8-dim group).
__device__ __forceinline__ void k_block(int b, int& key, int& dg) {
  const int col = b & 7, bis = (b >> 3) & 1, br = (b >> 4) & 15, sbc = b >> 8;
  key = sbc * 16 + bis * 8 + col;
  dg = br;
}
// Block b of a V tile: b_layout(V_t, 64, 128) -> (dim, 8-key group in tile).
__device__ __forceinline__ void v_block(int b, int& dim, int& kg) {
  const int col = b & 7, bis = (b >> 3) & 1, br = (b >> 4) & 7, sbc = b >> 7;
  dim = sbc * 16 + bis * 8 + col;
  kg = br;
}

__device__ __forceinline__ void put_block(uint8_t* dst, const uint16_t* src8) {
  const uint4 v = *reinterpret_cast<const uint4*>(src8);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t bits[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    bits[2 * i] = w[i] << 16;
    bits[2 * i + 1] = w[i] & 0xFFFF0000u;
  }
  uint32_t E, lo, hi, dq[4];
  bfp16_quant_block_fast(bits, E, lo, hi, dq);
  dst[0] = static_cast<uint8_t>(E);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    dst[1 + i] = static_cast<uint8_t>(lo >> (8 * i));
    dst[5 + i] = static_cast<uint8_t>(hi >> (8 * i));
  }
}

__device__ __forceinline__ void get_block(const uint8_t* src, uint16_t* dst8) {
  const uint32_t E = src[0];
  const uint32_t lo = src[1] | (src[2] << 8) | (src[3] << 16) | (static_cast<uint32_t>(src[4]) << 24);
  const uint32_t hi = src[5] | (src[6] << 8) | (src[7] << 16) | (static_cast<uint32_t>(src[8]) << 24);
  uint32_t w[4];
  bfp16_decode_block(E, lo, hi, w);
  *reinterpret_cast<uint4*>(dst8) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Q (H, T, tile) and KV (H, T, 2, tile) from q, k (H, 64T, 128) and vt (H, 128, ldv): one thread per block.
__global__ void __launch_bounds__(kThreads) pack_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                        const uint16_t* __restrict__ vt, int64_t ldv, int H, int T,
                                                        uint8_t* __restrict__ qo, uint8_t* __restrict__ kvo) {
  const int64_t per = static_cast<int64_t>(T) * kTileBlocks;       // blocks per head and stream
  const int64_t total = 3 * static_cast<int64_t>(H) * per;
  const int64_t rows = static_cast<int64_t>(T) * 64;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int s = static_cast<int>(i / (H * per));                  // 0 = Q, 1 = K, 2 = V
    const int64_t r = i % (H * per);
    const int h = static_cast<int>(r / per);
    const int t = static_cast<int>((r % per) / kTileBlocks), b = static_cast<int>(r % kTileBlocks);
    if (s == 0) {
      int row, dg;
      q_block(b, row, dg);
      put_block(qo + ((static_cast<int64_t>(h) * T + t) * kTileBlocks + b) * 9,
                q + (static_cast<int64_t>(h) * rows + 64 * t + row) * 128 + 8 * dg);
    } else if (s == 1) {
      int key, dg;
      k_block(b, key, dg);
      put_block(kvo + (((static_cast<int64_t>(h) * T + t) * 2 + 0) * kTileBlocks + b) * 9,
                k + (static_cast<int64_t>(h) * rows + 64 * t + key) * 128 + 8 * dg);
    } else {
      int dim, kg;
      v_block(b, dim, kg);
      put_block(kvo + (((static_cast<int64_t>(h) * T + t) * 2 + 1) * kTileBlocks + b) * 9,
                vt + (static_cast<int64_t>(h) * 128 + dim) * ldv + 64 * t + 8 * kg);
    }
  }
}

// Q tiles [t0, t0 + n) of each head (tpl tiles per head in the buffer) -> q (H, 64n, 128).
__global__ void __launch_bounds__(kThreads) q_unpack_kernel(const uint8_t* __restrict__ qi, int H, int tpl, int t0,
                                                            int n, uint16_t* __restrict__ q) {
  const int64_t per = static_cast<int64_t>(n) * kTileBlocks;
  const int64_t total = static_cast<int64_t>(H) * per;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int h = static_cast<int>(i / per);
    const int t = static_cast<int>((i % per) / kTileBlocks), b = static_cast<int>(i % kTileBlocks);
    int row, dg;
    q_block(b, row, dg);
    get_block(qi + ((static_cast<int64_t>(h) * tpl + t0 + t) * kTileBlocks + b) * 9,
              q + (static_cast<int64_t>(h) * n * 64 + 64 * t + row) * 128 + 8 * dg);
  }
}

// K / V tiles [t0, t0 + n) of each head's [K|V] tile sequence (tpl tiles per head) -> keys key0 + 64(t - t0) ..
// of k (H, nk, 128) and vt (H, 128, ldv).
__global__ void __launch_bounds__(kThreads) kv_unpack_kernel(const uint8_t* __restrict__ kvi, int H, int tpl, int t0,
                                                             int n, int64_t key0, int64_t nk, int64_t ldv,
                                                             uint16_t* __restrict__ k, uint16_t* __restrict__ vt) {
  const int64_t per = static_cast<int64_t>(n) * 2 * kTileBlocks;
  const int64_t total = static_cast<int64_t>(H) * per;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int h = static_cast<int>(i / per);
    const int64_t r = i % per;
    const int t = static_cast<int>(r / (2 * kTileBlocks));
    const int s = static_cast<int>((r / kTileBlocks) & 1), b = static_cast<int>(r % kTileBlocks);
    const uint8_t* src = kvi + (((static_cast<int64_t>(h) * tpl + t0 + t) * 2 + s) * kTileBlocks + b) * 9;
    const int64_t kb = key0 + 64 * t;
    if (s == 0) {
      int key, dg;
      k_block(b, key, dg);
      get_block(src, k + (static_cast<int64_t>(h) * nk + kb + key) * 128 + 8 * dg);
    } else {
      int dim, kg;
      v_block(b, dim, kg);
      get_block(src, vt + (static_cast<int64_t>(h) * 128 + dim) * ldv + kb + 8 * kg);
    }
  }
}

// The QKV table (T, 8448) bf16 -> cs (64T, 64, 2) = (cos, sin) per row and rotary pair, w_q, w_k (128 each).
// Entry j < 32 of block blk of tile t is cos at (row ROWS[blk][j / 4], pair PAIRS[blk][j % 4]), j >= 32 the sin of
// entry j - 32; ROWS[blk][a] = 16(blk / 32) + 8((blk % 4) / 2) + a, PAIRS[blk][b] = 8((blk / 4) % 8) + 4(blk % 2) + b.
__global__ void __launch_bounds__(kThreads) tables_kernel(const uint16_t* __restrict__ tab, int T,
                                                          float* __restrict__ cs, float* __restrict__ wq,
                                                          float* __restrict__ wk) {
  const int64_t total = static_cast<int64_t>(T) * 128 * 64;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int t = static_cast<int>(i / (128 * 64)), e = static_cast<int>(i % (128 * 64));
    const int blk = e >> 6, j = e & 63, jj = j & 31;
    const int row = 16 * (blk >> 5) + 8 * ((blk & 3) >> 1) + (jj >> 2);
    const int pair = 8 * ((blk >> 2) & 7) + 4 * (blk & 1) + (jj & 3);
    cs[((static_cast<int64_t>(t) * 64 + row) * 64 + pair) * 2 + (j >> 5)] =
        bf16_bits_to_float(tab[static_cast<int64_t>(t) * kTabRow + e]);
  }
  if (blockIdx.x == 0 && threadIdx.x < 128) {
    wq[threadIdx.x] = bf16_bits_to_float(tab[128 * 64 + threadIdx.x]);
    wk[threadIdx.x] = bf16_bits_to_float(tab[128 * 64 + 128 + threadIdx.x]);
  }
}

inline int grid_for(int64_t units) {
  const int64_t need = (units + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace npu
}  // namespace rl

extern "C" {

int rl_npu_qkv_pack(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int T,
                    uint8_t* q_out, uint8_t* kv_out, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(q && k && vt && q_out && kv_out, RL_ERR_ARGUMENT, "rl_npu_qkv_pack: NULL pointer");
  RL_REQUIRE(H > 0 && T > 0 && ldv >= 64LL * T && ldv % 8 == 0, RL_ERR_ARGUMENT,
             "rl_npu_qkv_pack: need H, T > 0 and ldv >= 64 T, ldv %% 8 == 0");
  RL_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(vt, 16), RL_ERR_ALIGNMENT,
             "rl_npu_qkv_pack: q, k, vt must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_npu_qkv_pack: needs an sm_100 device");
  const int64_t units = 3LL * H * T * npu::kTileBlocks;
  npu::pack_kernel<<<npu::grid_for(units), npu::kThreads, 0, stream>>>(q, k, vt, ldv, H, T, q_out, kv_out);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_npu_q_unpack(const uint8_t* q_in, int H, int tiles_per_head, int tile0, int ntiles, uint16_t* q,
                    rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(q_in && q, RL_ERR_ARGUMENT, "rl_npu_q_unpack: NULL pointer");
  RL_REQUIRE(H > 0 && ntiles > 0 && tile0 >= 0 && tile0 + ntiles <= tiles_per_head, RL_ERR_ARGUMENT,
             "rl_npu_q_unpack: tiles [%d, %d) outside %d per head", tile0, tile0 + ntiles, tiles_per_head);
  RL_REQUIRE(aligned(q, 16), RL_ERR_ALIGNMENT, "rl_npu_q_unpack: q must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_npu_q_unpack: needs an sm_100 device");
  const int64_t units = static_cast<int64_t>(H) * ntiles * npu::kTileBlocks;
  npu::q_unpack_kernel<<<npu::grid_for(units), npu::kThreads, 0, stream>>>(q_in, H, tiles_per_head, tile0, ntiles,
                                                                            q);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_npu_kv_unpack(const uint8_t* kv_in, int H, int tiles_per_head, int tile0, int ntiles, int64_t key0,
                     int64_t nk, int64_t ldv, uint16_t* k, uint16_t* vt, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(kv_in && k && vt, RL_ERR_ARGUMENT, "rl_npu_kv_unpack: NULL pointer");
  RL_REQUIRE(H > 0 && ntiles > 0 && tile0 >= 0 && tile0 + ntiles <= tiles_per_head, RL_ERR_ARGUMENT,
             "rl_npu_kv_unpack: tiles [%d, %d) outside %d per head", tile0, tile0 + ntiles, tiles_per_head);
  RL_REQUIRE(key0 >= 0 && key0 % 8 == 0 && key0 + 64LL * ntiles <= nk && nk <= ldv && ldv % 8 == 0,
             RL_ERR_ARGUMENT, "rl_npu_kv_unpack: keys [%lld, %lld) outside nk = %lld / ldv = %lld",
             static_cast<long long>(key0), static_cast<long long>(key0 + 64LL * ntiles), static_cast<long long>(nk),
             static_cast<long long>(ldv));
  RL_REQUIRE(aligned(k, 16) && aligned(vt, 16), RL_ERR_ALIGNMENT, "rl_npu_kv_unpack: k, vt must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_npu_kv_unpack: needs an sm_100 device");
  const int64_t units = static_cast<int64_t>(H) * ntiles * 2 * npu::kTileBlocks;
  npu::kv_unpack_kernel<<<npu::grid_for(units), npu::kThreads, 0, stream>>>(kv_in, H, tiles_per_head, tile0, ntiles,
                                                                             key0, nk, ldv, k, vt);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_npu_qkv_tables(const uint16_t* tables, int T, float* rope_cs, float* w_q, float* w_k, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(tables && rope_cs && w_q && w_k && T > 0, RL_ERR_ARGUMENT, "rl_npu_qkv_tables: bad arguments");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_npu_qkv_tables: needs an sm_100 device");
  npu::tables_kernel<<<npu::grid_for(static_cast<int64_t>(T) * 128 * 64), npu::kThreads, 0, stream>>>(
      tables, T, rope_cs, w_q, w_k);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

}  // extern "C"
