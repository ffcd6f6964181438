// Host-side helpers shared by the C-ABI translation units: error reporting and device queries.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/redline_b200.h"

namespace rl {

// Record a message for rl_last_error() (printf-style) and return `code`.
int fail(int code, const char* fmt, ...);
void clear_error();

// Multiprocessor count and compute capability of the current device (cached per device).
int sm_count();
bool device_is_sm100();

// cuTensorMapEncodeTiled, fetched from the driver through the runtime (no link-time libcuda dependency).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace rl

#define RL_TRY_CUDA(expr)                                                                     \
  do {                                                                                        \
    cudaError_t rl_e_ = (expr);                                                               \
    if (rl_e_ != cudaSuccess) return rl::fail(RL_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(rl_e_)); \
  } while (0)

#define RL_REQUIRE(cond, code, ...)               \
  do {                                            \
    if (!(cond)) return rl::fail(code, __VA_ARGS__); \
  } while (0)
