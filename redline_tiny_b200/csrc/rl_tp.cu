// Tensor-parallel reduction of the DiT's row-split projections, fused into the projection GEMM and the residual +
// LayerNorm kernel.
//
// The reference runs on one device; this library's tensor-parallel DiT (one reduction of the out- and
// down-projection partials per sublayer) needs
// every rank to form bf16(sum of the W partials) before the residual and LayerNorm. Here each rank's projection GEMM
// stores its bf16 partial, tile by tile as it is computed, into its own buffer and into the other rank's
// (rl_linear_bfp16_mirror over a CUDA IPC peer mapping), so the NVLink transfer overlaps the GEMM's math;
// rl_tp_signal then stores an epoch number into every rank's signal pad, and rl_ln_mod_tp waits (bounded) until the
// other ranks' epochs have arrived in its own pad and adds the W partials - now all in local memory - in rank order in
// fp32 inside the LayerNorm's first pass. No separate collective kernel runs.
//
// Protocol (per slot s, used alternately by the two projections of a block; epoch e increases by one per use):
//   GEMM -> partial[s][rank] here and in every other rank's buffer; rl_tp_signal(pads, W, rank, s, e):
//   pad_r[s][rank] = e on every rank r, after a system-scope fence; rl_ln_mod_tp(..., pad_self + s * W, e): waits for
//   pad_self[s][w] >= e for all w != rank, then reads partial[s][0..W-1].
// A rank stores into partial[s] again only after its next wait (on the other slot) has passed, which every other
// rank signals after it finished reading partial[s] (stream order on that rank), so the reads and the next stores of
// a slot never overlap.
#include "rl_common.cuh"
#include "rl_host.h"

#include <cstring>

namespace rl {
namespace tp {

__global__ void signal_kernel(unsigned long long* const* pads, int W, int rank, int slot, unsigned long long epoch) {
  const int r = threadIdx.x;
  if (r < W) {
    __threadfence_system();   // this rank's partial (written by the preceding kernels) before the flag
    unsigned long long* dst = pads[r] + static_cast<int64_t>(slot) * W + rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(epoch) : "memory");
  }
}

// One thread waits (bounded) until every other rank's entry of `pad` has reached `epoch`; the kernels after it on
// the stream start only when it ends. On timeout it records kErrWaitTimeout and returns.
__global__ void wait_kernel(const unsigned long long* pad, int W, int rank, unsigned long long epoch) {
  if (threadIdx.x != 0) return;
  for (int w = 0; w < W; ++w) {
    if (w == rank) continue;
    const long long t0 = clock64();
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(pad + w) : "memory");
      if (v >= epoch) break;
      if (clock64() - t0 > RL_WAIT_LIMIT_CYCLES) {
        report(kErrWaitTimeout);
        return;
      }
      __nanosleep(200);
    }
  }
}

}  // namespace tp
}  // namespace rl

extern "C" {

int rl_tp_signal(void* const* pads, int W, int rank, int slot, unsigned long long epoch, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(pads && W >= 1 && W <= 64 && rank >= 0 && rank < W && slot >= 0 && epoch > 0, RL_ERR_ARGUMENT,
             "rl_tp_signal: bad arguments");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_tp_signal: needs an sm_100 device");
  tp::signal_kernel<<<1, 64, 0, stream>>>(reinterpret_cast<unsigned long long* const*>(pads), W, rank, slot, epoch);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_ln_mod_tp(const uint16_t* x, const uint16_t* const* parts, int W, const unsigned long long* pad, int rank,
                 unsigned long long epoch, const uint16_t* params, int64_t M, int64_t D, int64_t row_split,
                 uint16_t* x_out, uint16_t* y_dq, uint8_t* y_q, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(x && parts && pad && params && W >= 1 && W <= 64 && rank >= 0 && rank < W && epoch > 0,
             RL_ERR_ARGUMENT, "rl_ln_mod_tp: bad arguments");
  RL_REQUIRE(M >= 0 && D >= 8 && D % 8 == 0, RL_ERR_ARGUMENT, "rl_ln_mod_tp: need D %% 8 == 0");
  RL_REQUIRE(aligned(x, 16) && aligned(params, 16) && aligned(x_out, 16) && aligned(y_dq, 16) && aligned(pad, 8),
             RL_ERR_ALIGNMENT, "rl_ln_mod_tp: bf16 pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_ln_mod_tp: needs an sm_100 device");
  if (M == 0) return RL_OK;
  return glue::launch_ln_mod(x, nullptr, 0, glue::TpBranch{parts, W}, pad, rank, epoch, params, M, D, row_split,
                             1e-6f, 0, x_out, y_dq, y_q, stream);
}

int rl_tp_wait(const unsigned long long* pad, int W, int rank, unsigned long long epoch, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(pad && W >= 1 && W <= 64 && rank >= 0 && rank < W && epoch > 0 && aligned(pad, 8), RL_ERR_ARGUMENT,
             "rl_tp_wait: bad arguments");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_tp_wait: needs an sm_100 device");
  tp::wait_kernel<<<1, 32, 0, stream>>>(pad, W, rank, epoch);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_ln_mod_tp_rs(const uint16_t* x, const uint16_t* const* parts, int W, const unsigned long long* pad, int rank,
                    unsigned long long epoch, const uint16_t* params, int64_t R, int64_t D, int64_t row_split,
                    uint16_t* x_out, uint16_t* const* y_dsts, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(x && parts && pad && params && x_out && y_dsts && W >= 1 && W <= 64 && rank >= 0 && rank < W &&
                 epoch > 0,
             RL_ERR_ARGUMENT, "rl_ln_mod_tp_rs: bad arguments");
  RL_REQUIRE(R >= 0 && R % 16 == 0 && D >= 8 && D % 8 == 0, RL_ERR_ARGUMENT,
             "rl_ln_mod_tp_rs: need R %% 16 == 0 and D %% 8 == 0");
  RL_REQUIRE(aligned(x, 16) && aligned(params, 16) && aligned(x_out, 16) && aligned(pad, 8) && aligned(y_dsts, 8),
             RL_ERR_ALIGNMENT, "rl_ln_mod_tp_rs: bf16 pointers must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_ln_mod_tp_rs: needs an sm_100 device");
  if (R == 0) return RL_OK;
  return glue::launch_ln_mod(x, nullptr, 0, glue::TpBranch{parts, W}, pad, rank, epoch, params, R, D, row_split,
                             1e-6f, 0, x_out, nullptr, nullptr, stream, glue::YPeers{y_dsts, W});
}

// Peer-readable buffers: a plain cudaMalloc allocation shared through a CUDA IPC handle (64 bytes), opened by the
// other ranks' processes as an ordinary peer mapping. The allocation is zeroed before it is returned, so the signal
// pads inside it start at epoch 0.
int rl_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  using namespace rl;
  RL_REQUIRE(ptr && handle && bytes > 0, RL_ERR_ARGUMENT, "rl_ipc_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  RL_TRY_CUDA(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    RL_TRY_CUDA(e);
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return RL_OK;
}

int rl_ipc_open(const void* handle, void** ptr) {
  using namespace rl;
  RL_REQUIRE(ptr && handle, RL_ERR_ARGUMENT, "rl_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  RL_TRY_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return RL_OK;
}

int rl_ipc_close(void* ptr) {
  using namespace rl;
  RL_REQUIRE(ptr, RL_ERR_ARGUMENT, "rl_ipc_close: null pointer");
  RL_TRY_CUDA(cudaIpcCloseMemHandle(ptr));
  return RL_OK;
}

int rl_ipc_free(void* ptr) {
  using namespace rl;
  RL_REQUIRE(ptr, RL_ERR_ARGUMENT, "rl_ipc_free: null pointer");
  RL_TRY_CUDA(cudaFree(ptr));
  return RL_OK;
}

}  // extern "C"
