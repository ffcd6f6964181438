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
// K and V tiles have separate three-stage pipelines: a K stage is released as soon as its QK product completes, so
// the producer keeps K loads about two blocks ahead of use (with one shared stage per block the load of block j+2
// could only start after P.V of block j-1, and it arrived late).
// Warp roles: warp 0 = TMA producer + TMEM allocator, warp 1 = MMA issuer (warp-wide loop, elected lane issues),
// warps 2-5 = softmax / correction / epilogue. O / l is rounded to bfp16 blocks of 8 along the head dim (the out-projection's A
// operand) and written row-major at columns h*128.. of the output.
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace attn {

constexpr int BQ = 128;                  // queries per CTA (TMEM lanes)
constexpr int HD = 128;                  // head dim
constexpr int BKV = 128;                 // keys per block
constexpr int SUB_ROWS_BYTES = 128;      // one swizzle row: 64 bf16
constexpr int kThreads = 192;            // producer, MMA issuer, 4 softmax warps
constexpr float kTau = 8.0f;             // lazy-rescale threshold (log2 units)
constexpr int kStages = 3;               // depth of each of the K and V pipelines
constexpr int Q_BYTES = BQ * HD * 2;     // two 128 x 64 sub-tiles
constexpr int K_SUB = BKV * SUB_ROWS_BYTES;
constexpr int K_BYTES = 2 * K_SUB;
constexpr int V_SUB = HD * SUB_ROWS_BYTES;   // 128 dims x 64 keys
constexpr int V_BYTES = (BKV / 64) * V_SUB;
constexpr int kQ = 0;
constexpr int kK = Q_BYTES;
constexpr int kV = kK + kStages * K_BYTES;
constexpr int kBar = kV + kStages * V_BYTES;
constexpr int kBytes = 1024 + kBar + 256;
constexpr int kTmemCols = 512;               // S buffers (2 x 128) + O (128), rounded to a power of two
constexpr int kOCol = 2 * BKV;
static_assert(kBytes <= 232448, "shared memory");

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

struct Params {
  int64_t Nq, Nk, nkv;
  int H;
  int kv_group;               // query heads per K/V head (grouped-query attention; 1 = one K/V head per query head)
  const int32_t* row_limit;   // per query row: last visible key (inclusive), or null
  float scale_log2;           // logits = (q . k) * scale_log2, in log2 units (> 0)
  uint16_t* o;
  float* o32;                 // when set: O / l written unrounded in fp32 here instead of bfp16-rounded bf16 to o
  int64_t ldo;
  int nblk;
};

// 2^x with the hardware approximation (MUFU.EX2); exp2(-inf) = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
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

// Bookkeeping of one load pipeline for the producer's error path: which stages have a load in flight, and the
// parity of its phase.
struct InFlight {
  uint32_t issued = 0, parity = 0;
  __device__ void note(int s, uint32_t ph) {
    issued |= 1u << s;
    parity = (parity & ~(1u << s)) | (ph << s);
  }
  __device__ void drain(uint64_t* full, int stages = kStages) const {
    for (int s = 0; s < stages; ++s)
      if (issued & (1u << s)) mbar_drain(&full[s], (parity >> s) & 1);
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kBar);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y;
  const int kvh = h / p.kv_group;   // the K/V head this query head reads
  const int nblk = p.nblk;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
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
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;   // S buffers: columns [0, 128), [128, 256); O: [256, 384)
  const uint32_t t_o = tmem + kOCol;

  if (warp == 0) {
    // ---------------- producer: Q, then K(t) and V(t - 1) in turn (K one block ahead of V) ----------------
    if (lane == 0) {
      bool ok = true;
      InFlight kf, vf;
      mbar_arrive_expect_tx(&bars->q_full, Q_BYTES);
      tma_load_3d(smem + kQ, &tm_q, &bars->q_full, 0, qt * BQ, h);
      tma_load_3d(smem + kQ + Q_BYTES / 2, &tm_q, &bars->q_full, 64, qt * BQ, h);
      for (int t = 0; ok && t <= nblk; ++t) {
        if (t < nblk) {
          const int s = t % kStages;
          const uint32_t ph = (t / kStages) & 1;
          if (!mbar_wait(&bars->k_empty[s], ph ^ 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->k_full[s], K_BYTES);
          uint8_t* kt = smem + kK + s * K_BYTES;
          tma_load_3d(kt, &tm_k, &bars->k_full[s], 0, t * BKV, kvh);
          tma_load_3d(kt + K_SUB, &tm_k, &bars->k_full[s], 64, t * BKV, kvh);
          kf.note(s, ph);
        }
        if (t >= 1) {
          const int j = t - 1, s = j % kStages;
          const uint32_t ph = (j / kStages) & 1;
          if (!mbar_wait(&bars->v_empty[s], ph ^ 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->v_full[s], V_BYTES);
          uint8_t* vt = smem + kV + s * V_BYTES;
          tma_load_3d(vt, &tm_v, &bars->v_full[s], j * BKV, 0, kvh);
          tma_load_3d(vt + V_SUB, &tm_v, &bars->v_full[s], j * BKV + 64, 0, kvh);
          vf.note(s, ph);
        }
      }
      if (!ok) {
        mbar_drain(&bars->q_full, 0);
        kf.drain(bars->k_full);
        vf.drain(bars->v_full);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop, one elected lane issues ----------------
    constexpr uint32_t idesc_s = idesc_bf16(BQ, BKV);   // S = Q K^T: M 128 (queries) x N 128 (keys)
    constexpr uint32_t idesc_o = idesc_bf16(BQ, HD);    // O += P V: M 128 (queries) x N 128 (dims)
    bool ok = true, any = false;
    const uint32_t qa = smem_u32(smem + kQ);
    auto issue_pv = [&](int jj) -> bool {
      const int sb = jj & 1, s = jj % kStages;
      if (!mbar_wait_warp(&bars->v_full[s], (jj / kStages) & 1, abort)) return false;
      if (!mbar_wait_warp(&bars->p_full[sb], (jj >> 1) & 1, abort)) return false;
      tc_fence_after();
      const uint32_t vb = smem_u32(smem + kV + s * V_BYTES);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k) {
          const uint64_t bdesc = sdesc_kmajor_sw128(vb + (k >> 2) * V_SUB) + 2 * (k & 3);
          umma_ts(t_o, tmem + sb * BKV + k * 8, bdesc, idesc_o, (jj | k) ? 1u : 0u);
        }
        umma_commit(&bars->v_empty[s]);
        umma_commit(&bars->pv_done[sb]);
      }
      __syncwarp();
      return true;
    };
    if (!mbar_wait_warp(&bars->q_full, 0, abort)) ok = false;
    for (int j = 0; ok && j < nblk; ++j) {
      const int s = j % kStages, sb = j & 1;
      if (!mbar_wait_warp(&bars->k_full[s], (j / kStages) & 1, abort)) { ok = false; break; }
      // S buffer sb is free once P.V of block j - 2 (which read P from it) has completed
      if (!mbar_wait_warp(&bars->pv_done[sb], ((j >> 1) & 1) ^ 1, abort)) { ok = false; break; }
      tc_fence_after();
      const uint32_t kb = smem_u32(smem + kK + s * K_BYTES);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t adesc = sdesc_kmajor_sw128(qa + (k >> 2) * (Q_BYTES / 2)) + 2 * (k & 3);
          const uint64_t bdesc = sdesc_kmajor_sw128(kb + (k >> 2) * K_SUB) + 2 * (k & 3);
          umma_ss(tmem + sb * BKV, adesc, bdesc, idesc_s, k ? 1u : 0u);
        }
        umma_commit(&bars->k_empty[s]);
        umma_commit(&bars->s_full[sb]);
      }
      __syncwarp();
      any = true;
      if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
    }
    if (ok && nblk > 0 && !issue_pv(nblk - 1)) ok = false;
    if (elect_one()) {
      if (ok) umma_commit(&bars->o_full);
      if (!ok && any) {
        umma_commit(&bars->drain);
        mbar_drain(&bars->drain, 0);
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax (warps 2-5; thread = query row = TMEM lane) ----------------
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
      uint32_t s[BKV];
      const uint32_t ta = tmem + sb * BKV + lane_off;
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t (&sc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32 * c]);
        RL_TMEM_LD32(ta + 32 * c, sc);
      }
      tmem_ld_wait_regs(s);
      // logits in log2 units, masked: key j*128 + c is visible iff key <= lim (lim < nkv); the maximum is taken on
      // the raw scores (scale_log2 > 0), masked entries set to -inf only in blocks that reach past lim
      const int64_t key0 = static_cast<int64_t>(j) * BKV;
      if (key0 + BKV - 1 > lim) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (key0 + c > lim) s[c] = 0xFF800000u;  // -inf
      }
      // row maximum as 8 independent chains of three-input max (one warp per SM sub-partition has no other work to
      // hide a 128-deep dependent chain behind)
      float mx;
      {
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = max3f(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]), -INFINITY);
#pragma unroll
        for (int c = 16; c < BKV; c += 16)
#pragma unroll
          for (int i = 0; i < 8; ++i) m8[i] = max3f(m8[i], __uint_as_float(s[c + 2 * i]), __uint_as_float(s[c + 2 * i + 1]));
        mx = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
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
      uint32_t pk[BKV / 2];
      float ls[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};   // 8 independent partial sums
      if (m_run == -INFINITY) {
#pragma unroll
        for (int c = 0; c < BKV / 2; ++c) pk[c] = 0u;
      } else {
        const float nm = -m_run, scl = p.scale_log2;
#pragma unroll
        for (int c = 0; c < BKV / 2; ++c) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * c]), scl, nm));
          const float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * c + 1]), scl, nm));
          pk[c] = pack_bf16x2(p0, p1);
          // the row sum adds the bf16 P that the P.V product multiplies (see softmax_block)
          ls[c & 7] += __uint_as_float(pk[c] << 16) + __uint_as_float(pk[c] & 0xFFFF0000u);
        }
      }
      l_run += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
#pragma unroll
      for (int c = 0; c < BKV / 64; ++c) {
        uint32_t (&pc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[32 * c]);
        RL_TMEM_ST32(ta + 32 * c, pc);
      }
      tmem_st_wait_regs(pk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[sb]);
    }
    // epilogue: O / l, rounded to bfp16 blocks of 8 along the head dim, row-major at columns h * 128
    if (ok && nblk > 0 && mbar_wait(&bars->o_full, 0, abort)) {
      tc_fence_after();
      const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      uint16_t* orow = p.o + qrow * p.ldo + static_cast<int64_t>(h) * HD;
      float* orow32 = p.o32 ? p.o32 + qrow * p.ldo + static_cast<int64_t>(h) * HD : nullptr;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        RL_TMEM_LD32(t_o + lane_off + 32 * c, o);
        tmem_ld_wait_regs(o);
        if (orow32) {
          if (qrow < p.Nq) {
#pragma unroll
            for (int b = 0; b < 8; ++b)
              reinterpret_cast<float4*>(orow32 + 32 * c + 4 * b)[0] =
                  make_float4(__uint_as_float(o[4 * b]) * inv, __uint_as_float(o[4 * b + 1]) * inv,
                              __uint_as_float(o[4 * b + 2]) * inv, __uint_as_float(o[4 * b + 3]) * inv);
          }
          continue;
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint32_t bits[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) bits[i] = __float_as_uint(__uint_as_float(o[8 * b + i]) * inv);
          uint32_t E, lo, hi, w[4];
          bfp16_quant_block_fast(bits, E, lo, hi, w);
          if (qrow < p.Nq) reinterpret_cast<uint4*>(orow + 32 * c + 8 * b)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// One 128-key block of the online softmax for the calling thread's query row (thread = TMEM lane): S is read from
// TMEM at `ta` (128 fp32 columns), masked past key `lim`, the running maximum raised lazily (by more than kTau), the
// thread's O row at `to` rescaled when it rises and `o_live` (a previous P.V has accumulated into it), and
// P = 2^(logit - m) written back over S as bf16 pairs, in two halves of 64 keys. The warp arrives on p_bar[0] once
// P is stored (kSplitP: on p_bar[0] after the first half and p_bar[1] after the second, so the MMA of the first
// half overlaps the exponentials of the second). Scaling and row sums use packed f32x2 arithmetic.
template <bool kSplitP>
__device__ __forceinline__ void softmax_block(uint32_t ta, uint32_t to, int64_t key0, int64_t lim, float scl,
                                              bool o_live, float& m_run, float& l_run, uint64_t* p_bar, int lane) {
  uint32_t s[BKV];
#pragma unroll
  for (int c = 0; c < BKV / 32; ++c) {
    uint32_t (&sc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32 * c]);
    RL_TMEM_LD32(ta + 32 * c, sc);
  }
  tmem_ld_wait_regs(s);
  if (key0 + BKV - 1 > lim) {
#pragma unroll
    for (int c = 0; c < BKV; ++c)
      if (key0 + c > lim) s[c] = 0xFF800000u;  // -inf
  }
  float mx;
  {
    float m8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m8[i] = max3f(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]), -INFINITY);
#pragma unroll
    for (int c = 16; c < BKV; c += 16)
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = max3f(m8[i], __uint_as_float(s[c + 2 * i]), __uint_as_float(s[c + 2 * i + 1]));
    mx = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
  }
  mx *= scl;
  const bool raise = mx > m_run + kTau;
  float alpha = 1.0f;
  if (raise) {
    alpha = exp2f(m_run - mx);
    l_run *= alpha;
    m_run = mx;
  }
  const bool rescale = o_live && __any_sync(0xffffffffu, raise);
  const bool none = m_run == -INFINITY;
  const float2 sc2 = make_float2(scl, scl), nm2 = make_float2(-m_run, -m_run);
  float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint32_t pk[32];
    if (none) {
#pragma unroll
      for (int c = 0; c < 32; ++c) pk[c] = 0u;
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int i = 64 * hh + 2 * c;
        const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[i]), __uint_as_float(s[i + 1])), sc2, nm2);
        const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
        pk[c] = pack_bf16x2(e.x, e.y);
        // the row sum adds the bf16 P that the P.V product multiplies, so that O / l weights V by exactly the
        // normalised P (a sum of the unrounded P would leave up to 2^-9 relative error in O where one key dominates)
        acc[c & 3] = __fadd2_rn(acc[c & 3], make_float2(__uint_as_float(pk[c] << 16),
                                                        __uint_as_float(pk[c] & 0xFFFF0000u)));
      }
    }
    RL_TMEM_ST32(ta + 32 * hh, pk);
    // rows whose running maximum rose rescale O (quiescent: the previous P.V completed before S was committed),
    // after the first half's exponentials so that the scores of that half no longer hold registers
    if (hh == 0 && rescale) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        RL_TMEM_LD32(to + 32 * c, o);
        tmem_ld_wait_regs(o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
        RL_TMEM_ST32(to + 32 * c, o);
        tmem_st_wait_regs(o);
      }
    }
    if (kSplitP || hh == 1) {
      tmem_st_wait_regs(pk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_bar[kSplitP ? hh : 0]);
    }
  }
  const float2 a01 = __fadd2_rn(acc[0], acc[1]), a23 = __fadd2_rn(acc[2], acc[3]);
  const float2 a = __fadd2_rn(a01, a23);
  l_run += a.x + a.y;
}

// O / l of the thread's query row, rounded to bfp16 blocks of 8 along the head dim, stored row-major.
__device__ __forceinline__ void store_o_row(uint32_t to, float l_run, uint16_t* orow, float* orow32, bool store) {
  const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t o[32];
    RL_TMEM_LD32(to + 32 * c, o);
    tmem_ld_wait_regs(o);
    if (orow32) {
      if (store) {
#pragma unroll
        for (int b = 0; b < 8; ++b)
          reinterpret_cast<float4*>(orow32 + 32 * c + 4 * b)[0] =
              make_float4(__uint_as_float(o[4 * b]) * inv, __uint_as_float(o[4 * b + 1]) * inv,
                          __uint_as_float(o[4 * b + 2]) * inv, __uint_as_float(o[4 * b + 3]) * inv);
      }
      continue;
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      uint32_t bits[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) bits[i] = __float_as_uint(__uint_as_float(o[8 * b + i]) * inv);
      uint32_t E, lo, hi, w[4];
      bfp16_quant_block_fast(bits, E, lo, hi, w);
      if (store) reinterpret_cast<uint4*>(orow + 32 * c + 8 * b)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Two query tiles per CTA (256 queries of one head). The MMA warp interleaves the tiles - P_0 V, S_0 = Q_0 K,
// P_1 V, S_1 = Q_1 K per key block - so the tensor pipe works on one tile while the other tile's softmax runs, and
// each K / V block is loaded once for both tiles. TMEM: S_0 [0, 128), S_1 [128, 256), O_0 [256, 384),
// O_1 [384, 512); P_t is written over S_t. S_t of the next block overwrites P_t, which P_t.V reads: kInOrder issues
// that Q.K right after the P.V - a write after a read by the MMA issued just before it on the same SM's tensor
// pipe, which executes one thread's MMAs in issue order, so the P.V's operand reads precede the Q.K's accumulator
// writes (the form every variant's outputs are compared against in the parity tests: they agree bit for bit) -
// otherwise the Q.K waits for the P.V's completion (one commit -> wake hand-off more per block, ~4 % slower).
// Warpgroup 0 (producer, MMA issuer, two idle warps) gives registers to the two softmax warpgroups (setmaxnreg):
// a softmax thread holds its 128 scores and 64 packed probabilities.
namespace two {
constexpr int kThreads = 384;
constexpr int KS = 3;                 // K pipeline depth
constexpr int VS = 2;                 // V pipeline depth
constexpr int kRegsLaunch = 168;      // registers per thread the kernel is launched with (65536 / 384, rounded to 8)
constexpr int kRegsLow = 80;          // warpgroup 0 after setmaxnreg.dec (the MMA issuer spills below 80)
constexpr int kRegsHigh = 208;        // softmax warpgroups after setmaxnreg.inc (no spills at 208)
static_assert(128 * kRegsLow + 256 * kRegsHigh <= kThreads * kRegsLaunch, "register split above the launch's total");
static_assert(kRegsLow + 2 * kRegsHigh <= 512, "register split above one SM sub-partition's file");
constexpr int kQ = 0;                 // Q_0, Q_1
constexpr int kK = 2 * Q_BYTES;
constexpr int kV = kK + KS * K_BYTES;
constexpr int kBar = kV + VS * V_BYTES;
constexpr int kBytes = 1024 + kBar + 256;
static_assert(kBytes <= 232448, "shared memory");

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[KS];
  uint64_t k_empty[KS];
  uint64_t v_full[VS];
  uint64_t v_empty[VS];
  uint64_t s_full[2];
  uint64_t p_full[2][2];   // [tile][half of P]; only [t][0] without kSplitP
  uint64_t pv_done[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

template <bool kInOrder, bool kSplitP>
__global__ void __launch_bounds__(kThreads, 1)
    attention2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kBar);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt2 = blockIdx.x, h = blockIdx.y;
  const int kvh = h / p.kv_group;
  const int nblk = p.nblk;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t][0], 4);
      mbar_init(&bars->p_full[t][1], 4);
      mbar_init(&bars->pv_done[t], 1);
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
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
  if (warp == 0) {
    // ---------------- producer: Q_0, Q_1, then K(t) and V(t - 1) in turn ----------------
    if (lane == 0) {
      bool ok = true;
      InFlight kf, vf;
      mbar_arrive_expect_tx(&bars->q_full, 2 * Q_BYTES);
      for (int t = 0; t < 2; ++t) {
        tma_load_3d(smem + kQ + t * Q_BYTES, &tm_q, &bars->q_full, 0, (2 * qt2 + t) * BQ, h);
        tma_load_3d(smem + kQ + t * Q_BYTES + Q_BYTES / 2, &tm_q, &bars->q_full, 64, (2 * qt2 + t) * BQ, h);
      }
      for (int t = 0; ok && t <= nblk; ++t) {
        if (t < nblk) {
          const int s = t % KS;
          const uint32_t ph = (t / KS) & 1;
          if (!mbar_wait(&bars->k_empty[s], ph ^ 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->k_full[s], K_BYTES);
          uint8_t* kt = smem + kK + s * K_BYTES;
          tma_load_3d(kt, &tm_k, &bars->k_full[s], 0, t * BKV, kvh);
          tma_load_3d(kt + K_SUB, &tm_k, &bars->k_full[s], 64, t * BKV, kvh);
          kf.note(s, ph);
        }
        if (t >= 1) {
          const int j = t - 1, s = j % VS;
          const uint32_t ph = (j / VS) & 1;
          if (!mbar_wait(&bars->v_empty[s], ph ^ 1, abort)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->v_full[s], V_BYTES);
          uint8_t* vt = smem + kV + s * V_BYTES;
          tma_load_3d(vt, &tm_v, &bars->v_full[s], j * BKV, 0, kvh);
          tma_load_3d(vt + V_SUB, &tm_v, &bars->v_full[s], j * BKV + 64, 0, kvh);
          vf.note(s, ph);
        }
      }
      if (!ok) {
        mbar_drain(&bars->q_full, 0);
        kf.drain(bars->k_full, KS);
        vf.drain(bars->v_full, VS);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (warp-wide, elected lane issues) ----------------
    constexpr uint32_t idesc_s = idesc_bf16(BQ, BKV);
    constexpr uint32_t idesc_o = idesc_bf16(BQ, HD);
    bool any = false;
    const uint32_t qa0 = smem_u32(smem + kQ);
    // S_t = Q_t K_j^T, once P_t of block j - 1 has been read by its P.V
    auto qk = [&](int t, int j) -> bool {
      const int s = j % KS;
      if (!mbar_wait_warp(&bars->k_full[s], (j / KS) & 1, abort)) return false;
      if (!kInOrder && j > 0 && !mbar_wait_warp(&bars->pv_done[t], (j - 1) & 1, abort)) return false;
      tc_fence_after();
      const uint32_t qa = qa0 + t * Q_BYTES;
      const uint32_t kb = smem_u32(smem + kK + s * K_BYTES);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t adesc = sdesc_kmajor_sw128(qa + (k >> 2) * (Q_BYTES / 2)) + 2 * (k & 3);
          const uint64_t bdesc = sdesc_kmajor_sw128(kb + (k >> 2) * K_SUB) + 2 * (k & 3);
          umma_ss(tmem + t * BKV, adesc, bdesc, idesc_s, k ? 1u : 0u);
        }
        umma_commit(&bars->s_full[t]);
        if (t == 1) umma_commit(&bars->k_empty[s]);
      }
      __syncwarp();
      any = true;
      return true;
    };
    // O_t += P_t V_j (kSplitP: the first 64 keys as soon as their half of P is stored)
    auto pv = [&](int t, int j) -> bool {
      const int s = j % VS;
      if (!mbar_wait_warp(&bars->v_full[s], (j / VS) & 1, abort)) return false;
      const uint32_t vb = smem_u32(smem + kV + s * V_BYTES);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (hh == 0 || kSplitP) {
          if (!mbar_wait_warp(&bars->p_full[t][hh], j & 1, abort)) return false;
          tc_fence_after();
        }
        if (elect_one()) {
#pragma unroll
          for (int k = 4 * hh; k < 4 * hh + 4; ++k) {
            const uint64_t bdesc = sdesc_kmajor_sw128(vb + (k >> 2) * V_SUB) + 2 * (k & 3);
            umma_ts(tmem + kOCol + t * HD, tmem + t * BKV + k * 8, bdesc, idesc_o, (j | k) ? 1u : 0u);
          }
          if (hh == 1) {
            if (!kInOrder) umma_commit(&bars->pv_done[t]);
            if (t == 1) umma_commit(&bars->v_empty[s]);
          }
        }
        __syncwarp();
      }
      return true;
    };
    bool ok = mbar_wait_warp(&bars->q_full, 0, abort) && qk(0, 0) && qk(1, 0);
    for (int j = 1; ok && j < nblk; ++j) ok = pv(0, j - 1) && qk(0, j) && pv(1, j - 1) && qk(1, j);
    if (ok) ok = pv(0, nblk - 1) && pv(1, nblk - 1);
    if (elect_one()) {
      if (ok) umma_commit(&bars->o_full);
      if (!ok && any) {
        umma_commit(&bars->drain);
        mbar_drain(&bars->drain, 0);
      }
    }
    __syncwarp();
  }
  } else {
    setmaxnreg_inc<kRegsHigh>();
    // ---------------- softmax of query tile t (thread = query row = TMEM lane) ----------------
    // S_t of block j is committed after P_t.V of block j - 1 was issued, so its arrival also means O_t is quiescent
    // and may be rescaled.
    const int t = (warp - 4) >> 2;
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const int64_t qrow = (static_cast<int64_t>(qt2) * 2 + t) * BQ + row;
    const uint32_t lane_off = (32u * q) << 16;
    const uint32_t ta = tmem + t * BKV + lane_off;
    const uint32_t to = tmem + kOCol + t * HD + lane_off;
    int64_t lim = p.nkv - 1;
    if (p.row_limit && qrow < p.Nq) lim = min(lim, static_cast<int64_t>(__ldg(p.row_limit + qrow)));
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!mbar_wait(&bars->s_full[t], j & 1, abort)) { ok = false; break; }
      tc_fence_after();
      softmax_block<kSplitP>(ta, to, static_cast<int64_t>(j) * BKV, lim, p.scale_log2, j > 0, m_run, l_run,
                             bars->p_full[t], lane);
    }
    if (ok && nblk > 0 && mbar_wait(&bars->o_full, 0, abort)) {
      tc_fence_after();
      const int64_t ooff = qrow * p.ldo + static_cast<int64_t>(h) * HD;
      store_o_row(to, l_run, p.o + ooff, p.o32 ? p.o32 + ooff : nullptr, qrow < p.Nq);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}
}  // namespace two

// Kernel choice for rl_attention_gqa: 0 = default (two query tiles per CTA, P released in halves, the next Q.K issued
// right behind the P.V: variant 5 - or the one-tile kernel when its grid needs fewer wave-cycles, as with the few
// heads per GPU of tensor parallelism), 1 = one tile per CTA; 2-5 = the two-tile forms 2 + 2 * kInOrder + kSplitP.
// Medians of 12 interleaved samples at config 3 (24 heads x 4352, B200): variant 2 240 us, 3 231 us, 4 226 us,
// 5 220 us (one tile per CTA: 257 us best case).
inline int& variant() {
  static int v = 0;
  return v;
}

// The two-tile kernel raises its softmax warpgroups' registers with setmaxnreg.inc, which waits until warpgroup 0
// has given enough back: that only ends if the kernel was compiled to launch with kRegsLaunch registers a thread.
template <bool kInOrder, bool kSplitP>
inline int two_tile_launch(dim3 grid, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                           const Params& p, cudaStream_t stream) {
  auto kern = two::attention2_kernel<kInOrder, kSplitP>;
  static int st = -1;
  static int regs = 0;
  if (st < 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess)
      return fail(RL_ERR_CUDA, "rl_attention: cudaFuncGetAttributes failed");
    regs = fa.numRegs;
    if (regs != two::kRegsLaunch) {
      st = RL_ERR_UNSUPPORTED;
    } else if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, two::kBytes) != cudaSuccess) {
      st = RL_ERR_CUDA;
    } else {
      st = RL_OK;
    }
  }
  if (st != RL_OK)
    return fail(st, "rl_attention: the two-tile kernel is unavailable (compiled with %d registers a thread, its "
                "register split needs %d, and 227 KB of shared memory)", regs, two::kRegsLaunch);
  kern<<<grid, two::kThreads, two::kBytes, stream>>>(mq, mk, mv, p);
  return RL_OK;
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

namespace rl {
namespace attn {

// The attention entry points: O / l rounded to bfp16 blocks of 8 as bf16 into o, or unrounded fp32 into o32.
int run(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int Hkv, int64_t Nq, int64_t Nk,
        int64_t nkv, const int32_t* row_limit, float scale_log2, uint16_t* o, float* o32, int64_t ldo,
        cudaStream_t stream) {
  RL_REQUIRE(q && k && vt && (o || o32), RL_ERR_ARGUMENT, "rl_attention: NULL pointer");
  RL_REQUIRE(H > 0 && Nq >= 0 && Nk > 0 && nkv >= 0 && nkv <= Nk && ldv >= Nk && ldv % 8 == 0, RL_ERR_ARGUMENT,
             "rl_attention: need 0 <= nkv <= Nk <= ldv, ldv %% 8 == 0");
  RL_REQUIRE(Hkv > 0 && H % Hkv == 0, RL_ERR_ARGUMENT, "rl_attention: %d query heads over %d K/V heads", H, Hkv);
  RL_REQUIRE(ldo >= static_cast<int64_t>(H) * HD && ldo % 8 == 0, RL_ERR_ARGUMENT,
             "rl_attention: ldo must be >= H * 128 and a multiple of 8");
  RL_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(vt, 16) && aligned(o, 16) && aligned(o32, 16) &&
                 aligned(row_limit, 4),
             RL_ERR_ALIGNMENT, "rl_attention: q, k, vt, o must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_attention: needs an sm_100 device");
  if (Nq == 0) return RL_OK;
  CUtensorMap mq, mk, mv;
  int st;
  if ((st = make_map(&mq, q, HD, Nq, H, HD * 2, Nq * HD * 2, 64, BQ)) != RL_OK) return st;
  if ((st = make_map(&mk, k, HD, Nk, Hkv, HD * 2, Nk * HD * 2, 64, BKV)) != RL_OK) return st;
  if ((st = make_map(&mv, vt, ldv, HD, Hkv, ldv * 2, ldv * HD * 2, 64, HD)) != RL_OK) return st;
  Params p;
  p.Nq = Nq;
  p.Nk = Nk;
  p.nkv = nkv;
  p.H = H;
  p.kv_group = H / Hkv;
  p.row_limit = row_limit;
  p.scale_log2 = scale_log2;
  p.o = o;
  p.o32 = o32;
  p.ldo = ldo;
  p.nblk = static_cast<int>((nkv + BKV - 1) / BKV);
  if (p.nblk == 0) {  // no visible key: the output is zero
    const size_t es = o32 ? 4 : 2;
    RL_TRY_CUDA(cudaMemset2DAsync(o32 ? static_cast<void*>(o32) : static_cast<void*>(o), ldo * es, 0,
                                  static_cast<size_t>(H) * HD * es, Nq, stream));
    return RL_OK;
  }
  int v = variant();
  if (v == 0) {
    // The two-tile kernel runs a key block of both tiles in ~3300 cycles, the one-tile kernel a key block of its tile
    // in ~2150 (clock64 traces at config 3); with few heads the two-tile grid fills a fraction of a wave, so take the
    // form with the fewer estimated wave-cycles.
    const int64_t sms = sm_count();
    const int64_t n2 = (Nq + 2 * BQ - 1) / (2 * BQ) * H, n1 = (Nq + BQ - 1) / BQ * H;
    if ((n1 + sms - 1) / sms * 2150 < (n2 + sms - 1) / sms * 3300) v = 1;
  }
  if (v != 1) {
    const dim3 grid(static_cast<unsigned>((Nq + 2 * BQ - 1) / (2 * BQ)), static_cast<unsigned>(H));
    switch (v) {
      case 2: st = two_tile_launch<false, false>(grid, mq, mk, mv, p, stream); break;
      case 3: st = two_tile_launch<false, true>(grid, mq, mk, mv, p, stream); break;
      case 4: st = two_tile_launch<true, false>(grid, mq, mk, mv, p, stream); break;
      case 5: st = two_tile_launch<true, true>(grid, mq, mk, mv, p, stream); break;
      default: st = two_tile_launch<true, true>(grid, mq, mk, mv, p, stream); break;
    }
    if (st != RL_OK) return st;
  } else {
    const dim3 grid(static_cast<unsigned>((Nq + BQ - 1) / BQ), static_cast<unsigned>(H));
    RL_TRY_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBytes));
    attention_kernel<<<grid, kThreads, kBytes, stream>>>(mq, mk, mv, p);
  }
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

}  // namespace attn
}  // namespace rl

extern "C" {

int rl_attention_gqa(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int Hkv,
                     int64_t Nq, int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, uint16_t* o,
                     int64_t ldo, rl_stream_t stream) {
  RL_REQUIRE(o, RL_ERR_ARGUMENT, "rl_attention: NULL pointer");
  return rl::attn::run(q, k, vt, ldv, H, Hkv, Nq, Nk, nkv, row_limit, scale_log2, o, nullptr, ldo, stream);
}

int rl_attention_gqa_f32(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int Hkv,
                         int64_t Nq, int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, float* o,
                         int64_t ldo, rl_stream_t stream) {
  RL_REQUIRE(o, RL_ERR_ARGUMENT, "rl_attention_gqa_f32: NULL pointer");
  return rl::attn::run(q, k, vt, ldv, H, Hkv, Nq, Nk, nkv, row_limit, scale_log2, nullptr, o, ldo, stream);
}

int rl_set_attention_variant(int variant) {
  const int prev = rl::attn::variant();
  rl::attn::variant() = variant;
  return prev;
}

int rl_attention(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int64_t ldv, int H, int64_t Nq,
                 int64_t Nk, int64_t nkv, const int32_t* row_limit, float scale_log2, uint16_t* o, int64_t ldo,
                 rl_stream_t stream) {
  return rl_attention_gqa(q, k, vt, ldv, H, H, Nq, Nk, nkv, row_limit, scale_log2, o, ldo, stream);
}

}  // extern "C"
