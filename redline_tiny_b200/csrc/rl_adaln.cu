// Per-step adaLN conditioning of the DiT on the GPU: timestep embedding, modulation and the bf16 parameter rows of
// the residual + LayerNorm kernel.
//
// Restates the reference's host glue (host_glue.py:31-48 and forward.py:231-238): for the rows [t, 0]
//   e   = [cos(1000 t f_i) | sin(1000 t f_i)], f_i = exp(-ln(10^4) i / 128), i < 128
//   te  = linear_2(SiLU(linear_1(e)))
//   mod = modulation(SiLU(te)) = [scale1 | gate1 | scale2 | gate2],  out = norm_out(SiLU(te))
// and the four LayerNorm parameter sets (rows [g | sc] per row group): first = (1, 1 + scale1),
// mlp = (tanh(gate1), 1 + scale2), attn = (tanh(gate2), 1 + scale1), out = (tanh(gate2), 1 + out), in bf16.
// The linears are fp32 matrix-vector products over at most four rows, HBM-bound on the weight (one warp per output
// column, 16-byte loads; the rows' inputs, after the optional SiLU, staged once per CTA in shared memory).
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace adaln {

constexpr int kThreads = 256;
constexpr int kMaxRows = 4;

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// y[r][n] = sum_k f(x[r][k]) w[n][k] (+ b[n]), r < R; f = SiLU when silu_in, else the identity.
__global__ void __launch_bounds__(kThreads) matvec_kernel(const float* __restrict__ w, int N, int K,
                                                          const float* __restrict__ x, int R,
                                                          const float* __restrict__ b, int silu_in,
                                                          float* __restrict__ y) {
  extern __shared__ float xs[];   // R x K
  for (int i = threadIdx.x; i < R * K; i += kThreads) {
    const float v = x[i];
    xs[i] = silu_in ? silu_f(v) : v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int n = blockIdx.x * (kThreads / 32) + warp; n < N; n += gridDim.x * (kThreads / 32)) {
    const float* wr = w + static_cast<int64_t>(n) * K;
    float acc[kMaxRows] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
    for (int k = 4 * lane; k < K; k += 128) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + k));
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        if (r < R) {
          const float4 xv = *reinterpret_cast<const float4*>(xs + r * K + k);
          acc[r] = fmaf(wv.x, xv.x, fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc[r]))));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    if (lane == 0) {
      const float bias = b ? b[n] : 0.0f;
      for (int r = 0; r < R; ++r) y[static_cast<int64_t>(r) * N + n] = acc[r] + bias;
    }
  }
}

// e[r] = [cos(t_r f_i) | sin(t_r f_i)] for the two rows t_0, t_1 (already scaled by 1000).
__global__ void sinusoidal_kernel(float t0, float t1, const float* __restrict__ freqs, int half,
                                  float* __restrict__ e) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * half) return;
  const int r = i / half, j = i % half;
  const float arg = (r ? t1 : t0) * freqs[j];
  e[r * 2 * half + j] = cosf(arg);
  e[r * 2 * half + half + j] = sinf(arg);
}

__global__ void params_kernel(const float* __restrict__ mod, const float* __restrict__ outs, int ld_out, int D,
                              uint16_t* __restrict__ first, uint16_t* __restrict__ mlp, uint16_t* __restrict__ attn,
                              uint16_t* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * D) return;
  const int r = i / D, d = i % D;
  const float* m = mod + static_cast<int64_t>(r) * 4 * D;
  const float s1 = m[d], g1 = m[D + d], s2 = m[2 * D + d], g2 = m[3 * D + d];
  const float os = outs[static_cast<int64_t>(r) * ld_out + d];
  const int64_t g = static_cast<int64_t>(r) * 2 * D + d, sc = g + D;
  const uint16_t tg2 = static_cast<uint16_t>(float_to_bf16_bits(tanhf(g2)));
  first[g] = 0x3F80;   // bf16 1.0
  first[sc] = static_cast<uint16_t>(float_to_bf16_bits(1.0f + s1));
  mlp[g] = static_cast<uint16_t>(float_to_bf16_bits(tanhf(g1)));
  mlp[sc] = static_cast<uint16_t>(float_to_bf16_bits(1.0f + s2));
  attn[g] = tg2;
  attn[sc] = static_cast<uint16_t>(float_to_bf16_bits(1.0f + s1));
  out[g] = tg2;
  out[sc] = static_cast<uint16_t>(float_to_bf16_bits(1.0f + os));
}

}  // namespace adaln
}  // namespace rl

extern "C" {

int rl_matvec_f32(const float* w, int N, int K, const float* x, int R, const float* bias, int silu_in, float* y,
                  rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(w && x && y, RL_ERR_ARGUMENT, "rl_matvec_f32: NULL pointer");
  RL_REQUIRE(N > 0 && K > 0 && K % 4 == 0 && R >= 1 && R <= adaln::kMaxRows, RL_ERR_ARGUMENT,
             "rl_matvec_f32: need N > 0, K %% 4 == 0, 1 <= R <= 4 (N=%d K=%d R=%d)", N, K, R);
  RL_REQUIRE(static_cast<int64_t>(R) * K * 4 <= 48 * 1024, RL_ERR_ARGUMENT, "rl_matvec_f32: R * K above 12288");
  RL_REQUIRE(aligned(w, 16) && aligned(x, 16) && aligned(bias, 4) && aligned(y, 4), RL_ERR_ALIGNMENT,
             "rl_matvec_f32: w and x must be 16-byte aligned");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_matvec_f32: needs an sm_100 device");
  const int per = adaln::kThreads / 32;
  const int grid = (N + per - 1) / per;
  adaln::matvec_kernel<<<grid, adaln::kThreads, static_cast<size_t>(R) * K * 4, stream>>>(w, N, K, x, R, bias,
                                                                                          silu_in ? 1 : 0, y);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_sinusoidal_embed(float t0, float t1, const float* freqs, int half, float* e, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(freqs && e && half > 0, RL_ERR_ARGUMENT, "rl_sinusoidal_embed: bad arguments");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_sinusoidal_embed: needs an sm_100 device");
  adaln::sinusoidal_kernel<<<(2 * half + 255) / 256, 256, 0, stream>>>(t0, t1, freqs, half, e);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

int rl_adaln_params(const float* mod, const float* out_scale, int ld_out, int D, uint16_t* first, uint16_t* mlp,
                    uint16_t* attn, uint16_t* out, rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(mod && out_scale && first && mlp && attn && out && D > 0 && ld_out >= D, RL_ERR_ARGUMENT,
             "rl_adaln_params: bad arguments");
  RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_adaln_params: needs an sm_100 device");
  adaln::params_kernel<<<(2 * D + 255) / 256, 256, 0, stream>>>(mod, out_scale, ld_out, D, first, mlp, attn, out);
  RL_TRY_CUDA(cudaGetLastError());
  return RL_OK;
}

}  // extern "C"
