// Shared device helpers for the redline B200 kernels (sm_100a only).
//
//  * status codes and the device-side error word every kernel reports into (never a trap or a device assert);
//  * bounded mbarrier waits: every spin on a barrier gives up after RL_WAIT_LIMIT_CYCLES, records an error and
//    lets the kernel drain and return;
//  * thin inline-PTX wrappers for TMA / bulk copies, mbarriers and the tcgen05 family (TMEM alloc, MMA, ld/st,
//    commit, fences);
//  * the bfp16 block codec shared by every kernel: one block = 8 values, 1 exponent byte E + 8 int8 mantissas,
//    value = m * 2^(E - 133).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/redline_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "redline_b200 is written for sm_100a only"
#endif

namespace rl {

// ------------------------------------------------------------------------------------------------------------
// device error word: bit flags OR-ed by kernels, read and cleared by rl_device_status()
// ------------------------------------------------------------------------------------------------------------
enum DeviceError : int {
  kErrWaitTimeout = 1,   // an mbarrier wait ran out of its cycle budget
  kErrBadArgument = 2,   // a kernel-side shape / index check failed (the access was skipped)
};

// Defined here: the library is one translation unit (redline_b200.cu includes every part).
__device__ int g_device_error = 0;

__device__ __forceinline__ void report(int code) { atomicOr(&g_device_error, code); }

// ~2 s at the B200's 1.9 GHz boost clock: far above any legitimate wait inside one launch.
constexpr long long RL_WAIT_LIMIT_CYCLES = 4000000000LL;

// ------------------------------------------------------------------------------------------------------------
// address helpers
// ------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the hardware suspend the thread until the phase completes or about `hint_ns` nanoseconds pass,
// so a waiting warp does not take issue slots from the warps that share its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `bar` with the given parity to complete. Gives up (returns false) when *abort is set by
// another role, or after RL_WAIT_LIMIT_CYCLES, in which case it sets *abort and reports kErrWaitTimeout. Each retry
// sleeps in hardware for at most ~0.5 ms, after which the abort flag and the limit are checked again.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 500000u)) return true;
    if (*abort) return false;
    if (clock64() - t0 > RL_WAIT_LIMIT_CYCLES) {
      *abort = 1;
      report(kErrWaitTimeout);
      return false;
    }
  }
}

// Short bounded wait used only on the error path, to let copies already in flight land before the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > 20000000LL) return;  // ~10 ms
  }
}

// ------------------------------------------------------------------------------------------------------------
// TMA and bulk copies (loads only, each into the issuing CTA's own shared memory)
// ------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Shared -> global bulk copy (16-byte aligned addresses, size a multiple of 16) in this thread's bulk group; the
// thread waits for its groups' shared-memory reads with bulk_store_wait_read before it rewrites the source.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, ld/st, fences (cta_group::1)
// ------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// True in exactly one lane of the (fully active) warp: the lowest, so repeated calls elect the same thread. MMA
// warps run their whole loop warp-wide (descriptors in uniform registers) and issue tcgen05.mma / commit from the
// elected lane: issued from divergent lane-0 code with per-thread descriptor registers, the MMA rate dropped to
// ~60% whenever another warp on the same SM sub-partition kept the FP32 pipe busy.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\telect.sync rx|px, %1;\n\tselp.b32 %0, 1, 0, px;\n\t}\n"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// Bounded wait taken by a whole warp; the outcome is made warp-uniform (false if any lane gave up).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulation.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T: the A operand (M rows = TMEM lanes, K packed two bf16 per column).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand stored with the 128-byte swizzle: rows of 64 bf16
// (128 B), 8-row groups 1024 B apart, 16-byte chunk c of row r at chunk position c ^ (r % 8). The tile base must be
// 1024-byte aligned. Advancing the start address by 32 B steps through K in slices of 16.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;           // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride byte offset: one 8-row group
  d |= static_cast<uint64_t>(1) << 46;           // descriptor version for tcgen05
  d |= static_cast<uint64_t>(2) << 61;           // SWIZZLE_128B
  return d;
}

// ------------------------------------------------------------------------------------------------------------
// CTA pairs: thread-block clusters of two CTAs on neighbouring SMs, tcgen05 with cta_group::2. Every tcgen05
// instruction of a kernel that uses these takes cta_group::2 (alloc / relinquish / dealloc by the same warp in both
// CTAs, MMA and commit by the leader CTA only).
// ------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address, in the cluster's shared window, of the variable at local shared address `saddr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Arrive on an mbarrier of any CTA in the cluster (default semantics: release at CTA scope). A cluster-scope release
// here cost 1000-1600 cycles per arrive on B200 and stalled every pipeline stage; the data the pair kernel hands over
// needs no more: decoded weights are read by their own CTA's tensor core (ordered by fence.proxy.async before the
// arrive), activation halves were written by TMA and completed on a barrier before the arrive, and TMEM hand-offs
// are ordered by the tcgen05 fences around the arrive and the wait.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// All threads of both CTAs of the cluster (every thread must reach it).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A * B^T over the pair: M = 256 (A rows 0-127 from the leader's shared memory, 128-255
// from the peer's, at the same offset), N columns of B split the same way, D rows in each CTA's own TMEM.
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// As umma_ss_pair with A from tensor memory: each CTA's A rows sit in its own TMEM at the same address.
__device__ __forceinline__ void umma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at `cluster_addr` (either CTA of the pair) when every pair MMA issued so far by this
// thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

#define RL_TMEM_LD32(taddr, r)                                                                                   \
  asm volatile(                                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"  \
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                        \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),          \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),    \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),  \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])   \
      : "r"(taddr))

#define RL_TMEM_ST32(taddr, r)                                                                                   \
  asm volatile(                                                                                                  \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"   \
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                         \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),          \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), \
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),            \
      "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]))

#define RL_TMEM_LD16(taddr, r)                                                                                   \
  asm volatile(                                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"   \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),          \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])     \
      : "r"(taddr))

#define RL_TMEM_ST16(taddr, r)                                                                                   \
  asm volatile(                                                                                                  \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" :: \
      "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),          \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]))

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// tcgen05.ld writes its destination registers asynchronously: the wait names them as read-write operands so the
// compiler cannot move a use of the loaded values above it. Likewise a store's source registers stay live (and
// unmodified) until its wait.
template <int N>
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}
template <int N>
__device__ __forceinline__ void tmem_st_wait_regs(const uint32_t (&r)[N]) {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" ::"r"(r[i]) : "memory");
}

// ------------------------------------------------------------------------------------------------------------
// bfp16 codec
// ------------------------------------------------------------------------------------------------------------

// Quantise 8 float32 values (given as raw bits) into one block: E = largest exponent field; each mantissa is the
// 24-bit significand shifted right by 17 + E - max(e, 1), rounded half to even, signed, clipped to [-128, 127].
// This is exactly rint(x * 2^(133 - E)) computed without forming 2^(133 - E) (which overflows float32 for small E).
__device__ __forceinline__ uint32_t bfp16_block_exponent(const uint32_t (&b)[8]) {
  uint32_t e = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) e = max(e, (b[i] >> 23) & 0xFFu);
  return e;
}

__device__ __forceinline__ int bfp16_quant_one(uint32_t bits, uint32_t E) {
  const uint32_t field = (bits >> 23) & 0xFFu;
  const uint32_t sig = field ? ((bits & 0x7FFFFFu) | 0x800000u) : (bits & 0x7FFFFFu);
  const uint32_t shift = 17u + E - (field ? field : 1u);   // >= 16
  int q;
  if (shift > 25u) {
    q = 0;
  } else {
    const uint32_t t = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    q = static_cast<int>(t + ((rem > half) || (rem == half && (t & 1u))));
  }
  q = (bits >> 31) ? -q : q;
  return max(-128, min(127, q));
}

// Quantise one block and decode it again, with float arithmetic (the fast path of the quantiser kernels).
// E = (max |bits|) >> 23 is the largest exponent field. For E >= 7, s = 2^(133-E) is a normal float and
// fma(x, s, 1.5 * 2^23) = 1.5 * 2^23 + rint_half_even(x * s) exactly (the product is exact inside the FMA and
// |x * s| < 256, so the one rounding of the sum is the round-half-even of x * s); the mantissa is clamped to
// [-128, 127] in float, its low byte read from the bits of m + 1.5 * 2^23, and the decoded value is m * 2^(E-133).
// Blocks with E < 7 (every value below 2^-120) take the exact integer path above.
__device__ __forceinline__ void bfp16_quant_block_fast(const uint32_t (&b)[8], uint32_t& E, uint32_t& lo,
                                                       uint32_t& hi, uint32_t (&dq)[4]);

// 2^(E - 133) as float32 bits (subnormal for E < 7).
__device__ __forceinline__ float bfp16_scale(uint32_t E) {
  return __uint_as_float(E >= 7u ? ((E - 6u) << 23) : (1u << (E + 16u)));
}

// Decode one block whose 8 mantissas are given in offset binary (byte i of u0 = m_i + 128, byte i of u1 =
// m_{4+i} + 128) into four bf16x2 words (low half = even element). Exact: m * 2^(E-133) has <= 8 significant bits,
// so its float32 form has zero low 16 bits and the top half is the bf16 value. Fast path (7 <= E <= 237): with
// s = 2^(E-133) built by one integer multiply-add, v = (2^23 + u) * s - (2^23 + 128) * s in a single FMA is exact
// because the result is representable and (2^23 + 128) * s is finite. Other exponents take a plain multiply.
__device__ __forceinline__ void bfp16_decode_block_ob(uint32_t E, uint32_t u0, uint32_t u1, uint32_t (&w)[4]) {
  float v[8];
  if (E - 7u <= 230u) {
    const float s = __uint_as_float(E * 0x800000u - 0x3000000u);
    const float c = -8388736.0f * s;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = fmaf(__uint_as_float(__byte_perm(u0, 0x4B000000u, 0x7540u + i)), s, c);
      v[4 + i] = fmaf(__uint_as_float(__byte_perm(u1, 0x4B000000u, 0x7540u + i)), s, c);
    }
  } else {
    const float s = bfp16_scale(E);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __fmul_rn(static_cast<float>(static_cast<int>((u0 >> (8 * i)) & 0xFFu) - 128), s);
      v[4 + i] = __fmul_rn(static_cast<float>(static_cast<int>((u1 >> (8 * i)) & 0xFFu) - 128), s);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = __byte_perm(__float_as_uint(v[2 * i]), __float_as_uint(v[2 * i + 1]), 0x7632u);
}

// The same for two's-complement mantissa bytes (the bfp16 stream format).
__device__ __forceinline__ void bfp16_decode_block(uint32_t E, uint32_t lo, uint32_t hi, uint32_t (&w)[4]) {
  bfp16_decode_block_ob(E, lo ^ 0x80808080u, hi ^ 0x80808080u, w);
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ void bfp16_quant_block_fast(const uint32_t (&b)[8], uint32_t& E, uint32_t& lo,
                                                       uint32_t& hi, uint32_t (&dq)[4]) {
  uint32_t mx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) mx = max(mx, b[i] & 0x7FFFFFFFu);
  E = mx >> 23;
  if (E >= 7u) {
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    const float s = __uint_as_float((260u - E) << 23);
    const float inv = __uint_as_float((E - 6u) << 23);
    uint32_t byte[8];
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = fmaf(__uint_as_float(b[i]), s, kMagic);
      const float m = fminf(fmaxf(__fsub_rn(y, kMagic), -128.0f), 127.0f);
      byte[i] = __float_as_uint(__fadd_rn(m, kMagic)) & 0xFFu;
      v[i] = __fmul_rn(m, inv);
    }
    lo = byte[0] | (byte[1] << 8) | (byte[2] << 16) | (byte[3] << 24);
    hi = byte[4] | (byte[5] << 8) | (byte[6] << 16) | (byte[7] << 24);
#pragma unroll
    for (int i = 0; i < 4; ++i) dq[i] = __byte_perm(__float_as_uint(v[2 * i]), __float_as_uint(v[2 * i + 1]), 0x7632u);
  } else {
    lo = hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo |= (static_cast<uint32_t>(bfp16_quant_one(b[i], E)) & 0xFFu) << (8 * i);
      hi |= (static_cast<uint32_t>(bfp16_quant_one(b[4 + i], E)) & 0xFFu) << (8 * i);
    }
    bfp16_decode_block(E, lo, hi, dq);
  }
}

// float32 -> bf16 bits, round half to even (finite inputs).
__device__ __forceinline__ uint32_t float_to_bf16_bits(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b + 0x7FFFu + ((b >> 16) & 1u)) >> 16;
}

}  // namespace rl
