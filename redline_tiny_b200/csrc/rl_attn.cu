// Joint text+image flash attention on tcgen05 (sm_100a), head_dim 128.
//
// Restates the reference's attention (kernels/attn/attn_bfp.cc: attn_qk / attn_pv / attn_end_a, lines 846-923, with
// the key-tail mask of lines 252-270 and the per-row key limits of lines 642-662): softmax(Q K^T) V per head with an
// online softmax in the exp2 domain and a lazy rescale (the running maximum is only raised when a block's maximum
// exceeds it by more than TAU = 8, so the accumulator is rarely rescaled). Unlike the NPU, P is kept in bf16 and O
// accumulates in fp32.
//
// One CTA per (128-query tile, head). Per 128-key block j:
//   S_j = Q K_j^T        tcgen05.mma M128 N128, both operands K-major in shared memory (TMA, 128-byte swizzle),
//                        fp32 into one of two TMEM S buffers (double-buffered: QK of block j+1 overlaps softmax j);
//   softmax              4 warps, thread = query row = TMEM lane: tcgen05.ld of the row, mask, max, exp2, row sum;
//                        P (bf16) written back over the same TMEM columns with tcgen05.st;
//   O += P_j V_j         tcgen05.mma with A = P from TMEM, B = V^T (dims x keys, keys contiguous) in shared memory.
// Warp roles: warp 0 = TMA producer + TMEM allocator, warp 1 = MMA issuer, warps 4-7 = softmax / correction /
// epilogue. O / l is rounded to bfp16 blocks of 8 along the head dim (the out-projection's A operand) and written
// row-major at columns h*128.. of the output.
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace attn {

constexpr int BQ = 128;                  // queries per CTA (TMEM lanes)
constexpr int BKV = 128;                 // keys per block
constexpr int HD = 128;                  // head dim
constexpr int HALF_BYTES = 128 * 64 * 2; // one 128-row x 64-element SW128 sub-tile (16 KB)
constexpr int TILE_BYTES = 2 * HALF_BYTES;
constexpr int kStages = 3;               // K/V stages
constexpr int kThreads = 256;
constexpr float kTau = 8.0f;             // lazy-rescale threshold (log2 units)

struct Smem {
  // 1024-aligned tiles: Q, then per stage K and V^T
  static constexpr int kQ = 0;
  static constexpr int kK = TILE_BYTES;
  static constexpr int kV = kK + kStages * TILE_BYTES;
  static constexpr int kBar = kV + kStages * TILE_BYTES;
  static constexpr int kBytes = 1024 + kBar + 256;
};
static_assert(Smem::kBytes <= 232448, "shared memory");

struct Barriers {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  int64_t Nq, Nk, nkv;
  int H;
  const int32_t* row_limit;   // per query row: last visible key (inclusive), or null
  float scale_log2;           // logits = (q . k) * scale_log2, in log2 units
  uint16_t* o;
  int64_t ldo;
  int nblk;
};

// 2^x with the hardware approximation (MUFU.EX2); exp2(-inf) = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two floats -> bf16x2 (round to nearest even), low half = a.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + Smem::kBar);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y;
  const int nblk = p.nblk;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 4);
      mbar_init(&bars->pv_done[b], 1);
    }
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;   // S buffers: columns [0,128), [128,256); O: [256, 384)
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      bool ok = true;
      uint32_t issued = 0, last_par = 0;
      mbar_arrive_expect_tx(&bars->q_full, TILE_BYTES);
      tma_load_3d(smem + Smem::kQ, &tm_q, &bars->q_full, 0, qt * BQ, h);
      tma_load_3d(smem + Smem::kQ + HALF_BYTES, &tm_q, &bars->q_full, 64, qt * BQ, h);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&bars->kv_empty[s], ph ^ 1, abort)) { ok = false; break; }
        mbar_arrive_expect_tx(&bars->kv_full[s], 2 * TILE_BYTES);
        uint8_t* kt = smem + Smem::kK + s * TILE_BYTES;
        uint8_t* vt = smem + Smem::kV + s * TILE_BYTES;
        tma_load_3d(kt, &tm_k, &bars->kv_full[s], 0, j * BKV, h);
        tma_load_3d(kt + HALF_BYTES, &tm_k, &bars->kv_full[s], 64, j * BKV, h);
        tma_load_3d(vt, &tm_v, &bars->kv_full[s], j * BKV, 0, h);
        tma_load_3d(vt + HALF_BYTES, &tm_v, &bars->kv_full[s], j * BKV + 64, 0, h);
        issued |= 1u << s;
        last_par = (last_par & ~(1u << s)) | (ph << s);
      }
      if (!ok) {
        mbar_drain(&bars->q_full, 0);
        for (int s = 0; s < kStages; ++s)
          if (issued & (1u << s)) mbar_drain(&bars->kv_full[s], (last_par >> s) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BQ, BKV);
      bool ok = true, any = false;
      const uint32_t qa = smem_u32(smem + Smem::kQ);
      auto issue_pv = [&](int jj) -> bool {
        const int sb = jj & 1, s = jj % kStages;
        if (!mbar_wait(&bars->p_full[sb], (jj >> 1) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(smem + Smem::kV + s * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k) {
          const uint64_t bdesc = sdesc_kmajor_sw128(vb + (k >> 2) * HALF_BYTES) + 2 * (k & 3);
          umma_ts(t_o, tmem + sb * 128 + k * 8, bdesc, idesc, (jj | k) ? 1u : 0u);
        }
        umma_commit(&bars->kv_empty[s]);
        umma_commit(&bars->pv_done[sb]);
        return true;
      };
      if (!mbar_wait(&bars->q_full, 0, abort)) ok = false;
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % kStages, sb = j & 1;
        if (!mbar_wait(&bars->kv_full[s], (j / kStages) & 1, abort)) { ok = false; break; }
        // S buffer sb is free once PV of block j - 2 (which read P from it) has completed
        if (!mbar_wait(&bars->pv_done[sb], ((j >> 1) & 1) ^ 1, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t kb = smem_u32(smem + Smem::kK + s * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t adesc = sdesc_kmajor_sw128(qa + (k >> 2) * HALF_BYTES) + 2 * (k & 3);
          const uint64_t bdesc = sdesc_kmajor_sw128(kb + (k >> 2) * HALF_BYTES) + 2 * (k & 3);
          umma_ss(tmem + sb * 128, adesc, bdesc, idesc, k ? 1u : 0u);
        }
        any = true;
        umma_commit(&bars->s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && nblk > 0 && !issue_pv(nblk - 1)) ok = false;
      if (ok) umma_commit(&bars->o_full);
      if (!ok && any) {
        umma_commit(&bars->drain);
        mbar_drain(&bars->drain, 0);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax (thread = query row) ----------------
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const int64_t qrow = static_cast<int64_t>(qt) * BQ + row;
    const uint32_t lane_off = (32u * q) << 16;
    int64_t lim = p.nkv - 1;
    if (p.row_limit && qrow < p.Nq) lim = min(lim, static_cast<int64_t>(__ldg(p.row_limit + qrow)));
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&bars->s_full[sb], (j >> 1) & 1, abort)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
      {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
        uint32_t (&s2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[64]);
        uint32_t (&s3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[96]);
        const uint32_t ta = tmem + sb * 128 + lane_off;
        RL_TMEM_LD32(ta, s0);
        RL_TMEM_LD32(ta + 32, s1);
        RL_TMEM_LD32(ta + 64, s2);
        RL_TMEM_LD32(ta + 96, s3);
        tmem_ld_wait_regs(s);
      }
      // logits in log2 units, masked: key j*128 + c is visible iff key <= lim (lim < nkv); the maximum is taken on
      // the raw scores (scale_log2 > 0), masked entries set to -inf only in blocks that reach past lim
      const int64_t key0 = static_cast<int64_t>(j) * BKV;
      float mx = -INFINITY;
      if (key0 + BKV - 1 <= lim) {
#pragma unroll
        for (int c = 0; c < 128; ++c) mx = fmaxf(mx, __uint_as_float(s[c]));
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (key0 + c > lim) s[c] = 0xFF800000u;  // -inf
          mx = fmaxf(mx, __uint_as_float(s[c]));
        }
      }
      mx *= p.scale_log2;
      const bool raise = mx > m_run + kTau;      // true on the first block with any visible key
      float alpha = 1.0f;
      if (raise) {
        alpha = exp2f(m_run - mx);               // 0 when m_run is -inf
        l_run *= alpha;
        m_run = mx;
      }
      // rows whose running maximum rose rescale their slice of O, once the previous P.V has landed in it
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        if (!mbar_wait(&bars->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          RL_TMEM_LD32(t_o + lane_off + 32 * c, o);
          tmem_ld_wait_regs(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          RL_TMEM_ST32(t_o + lane_off + 32 * c, o);
          tmem_st_wait_regs(o);
        }
      }
      // P = 2^(logit - m_run) with the hardware exp2 (P is stored as bf16 anyway), written over S
      uint32_t pk[64];
      float lsum = 0.0f;
      if (m_run == -INFINITY) {
#pragma unroll
        for (int c = 0; c < 64; ++c) pk[c] = 0u;
      } else {
        const float nm = -m_run, sc = p.scale_log2;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * c]), sc, nm));
          const float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * c + 1]), sc, nm));
          lsum += p0 + p1;
          pk[c] = pack_bf16x2(p0, p1);
        }
      }
      l_run += lsum;
      {
        uint32_t (&p0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[0]);
        uint32_t (&p1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[32]);
        const uint32_t ta = tmem + sb * 128 + lane_off;
        RL_TMEM_ST32(ta, p0);
        RL_TMEM_ST32(ta + 32, p1);
        tmem_st_wait_regs(pk);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[sb]);
    }
    // epilogue: O / l, rounded to bfp16 blocks of 8 along the head dim, row-major at columns h * 128
    if (ok && nblk > 0 && mbar_wait(&bars->o_full, 0, abort)) {
      tc_fence_after();
      const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      uint16_t* orow = p.o + qrow * p.ldo + static_cast<int64_t>(h) * HD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        RL_TMEM_LD32(t_o + lane_off + 32 * c, o);
        tmem_ld_wait_regs(o);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint32_t bits[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) bits[i] = __float_as_uint(__uint_as_float(o[8 * b + i]) * inv);
          const uint32_t E = bfp16_block_exponent(bits);
          uint32_t lo = 0, hi = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            lo |= (static_cast<uint32_t>(bfp16_quant_one(bits[i], E)) & 0xFFu) << (8 * i);
            hi |= (static_cast<uint32_t>(bfp16_quant_one(bits[4 + i], E)) & 0xFFu) << (8 * i);
          }
          uint32_t w[4];
          bfp16_decode_block(E, lo, hi, w);
          if (qrow < p.Nq) reinterpret_cast<uint4*>(orow + 32 * c + 8 * b)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        }
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

inline int make_map(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                    uint64_t stride2, uint32_t b0, uint32_t b1) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(RL_ERR_CUDA, "rl_attention: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t gdim[3] = {d0, d1, d2};
  const cuuint64_t gstride[2] = {stride1, stride2};
  const cuuint32_t box[3] = {b0, b1, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RL_ERR_CUDA, "rl_attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return RL_OK;
}

}  // namespace attn
}  // namespace rl

extern "C" {

int rl_attention(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int64_t Nq,
                 int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, uint16_t* o, int64_t ldo,
                 rl_stream_t stream) {
  using namespace rl;
  using namespace rl::attn;
  RL_REQUIRE(q && k && vt && o, RL_ERR_ARGUMENT, "rl_attention: NULL pointer");
  RL_REQUIRE(H > 0 && Nq >= 0 && Nk > 0 && nkv >= 0 && nkv <= Nk && ldv >= Nk && ldv % 8 == 0, RL_ERR_ARGUMENT,
             "rl_attention: need 0 <= nkv <= Nk <= ldv, ldv %% 8 == 0");
  RL_REQUIRE(ldo >= static_cast<int64_t>(H) * HD && ldo % 8 == 0, RL_ERR_ARGUMENT,
             "rl_attention: ldo must be >= H * 128 and a multiple of 8");
  RL_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(vt, 16) && aligned(o, 16) && aligned(row_limit, 4),
             RL_ERR_ALIGNMENT, "rl_attention: q, k, vt, o must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_attention: needs an sm_100 device");
  if (Nq == 0) return RL_OK;
  CUtensorMap mq, mk, mv;
  int st;
  if ((st = make_map(&mq, q, HD, Nq, H, HD * 2, Nq * HD * 2, 64, BQ)) != RL_OK) return st;
  if ((st = make_map(&mk, k, HD, Nk, H, HD * 2, Nk * HD * 2, 64, BKV)) != RL_OK) return st;
  if ((st = make_map(&mv, vt, ldv, HD, H, ldv * 2, ldv * HD * 2, 64, HD)) != RL_OK) return st;
  Params p;
  p.Nq = Nq;
  p.Nk = Nk;
  p.nkv = nkv;
  p.H = H;
  p.row_limit = row_limit;
  p.scale_log2 = scale_log2;
  p.o = o;
  p.ldo = ldo;
  p.nblk = static_cast<int>((nkv + BKV - 1) / BKV);
  if (p.nblk == 0) {  // no visible key: the output is zero
    RL_TRY_CUDA(cudaMemset2DAsync(o, ldo * 2, 0, static_cast<size_t>(H) * HD * 2, Nq, stream));
    return RL_OK;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    RL_TRY_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::kBytes));
    attr_set[dev] = true;
  }
  const dim3 grid(static_cast<unsigned>((Nq + BQ - 1) / BQ), static_cast<unsigned>(H));
  attention_kernel<<<grid, kThreads, Smem::kBytes, stream>>>(mq, mk, mv, p);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

}  // extern "C"
