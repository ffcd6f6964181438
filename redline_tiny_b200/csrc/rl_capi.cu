// Library-wide C ABI: errors, version, device status; plus the host helpers declared in rl_host.h.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {

static thread_local char t_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_last_error[0] = '\0'; }

namespace {
constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices] = {0};
int g_major[kMaxDevices] = {0};
std::mutex g_mu;

void query(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[dev]) return;
  int sms = 0, major = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  g_major[dev] = major;
  g_sms[dev] = sms > 0 ? sms : 1;
}
}  // namespace

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return 1;
  query(dev);
  return g_sms[dev];
}

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
  query(dev);
  return g_major[dev] == 10;
}

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace rl

extern "C" {

const char* rl_last_error(void) { return rl::t_last_error; }

int rl_version(void) { return 100; }

int rl_device_status(int* flags_out) {
  RL_TRY_CUDA(cudaDeviceSynchronize());
  int flags = 0;
  RL_TRY_CUDA(cudaMemcpyFromSymbol(&flags, rl::g_device_error, sizeof(int)));
  const int zero = 0;
  RL_TRY_CUDA(cudaMemcpyToSymbol(rl::g_device_error, &zero, sizeof(int)));
  if (flags_out) *flags_out = flags;
  if (flags) return rl::fail(RL_ERR_DEVICE, "device error flags 0x%x (1: wait timeout, 2: range check)", flags);
  return RL_OK;
}

}  // extern "C"
