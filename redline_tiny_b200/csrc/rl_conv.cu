// VAE decoder convolution (3x3 pad 1, or 1x1; stride 1) with bfp16 weights, as a GEMM on the packed-weight kernel.
//
// Restates the reference's vconv (kernels/vae/vconv.cc:1-17, weights packed by redline/vae_ops.py:44-61
// pack_vconv, checked against vae_ops.conv_ref, vae_ops.py:64-75): out[y][x][co] = b[co] +
// sum_{dy,dx,ci} in[y+dy-1][x+dx-1][ci] * w[co][ci][dy][dx]. The reference quantises its weights to bfp16 blocks of
// 8 input channels per (output channel, tap) and its activation strips to bfp16 blocks of 8 channels per pixel; here
// the weights are the GEMM's B = [(dy, dx, ci)][co] in the native tile format (blocks of 8 along K = 8 input
// channels of one tap: the same blocks; each tap's channels are padded with zero rows to a multiple of 64, the
// kernel's K step), and the activations are the quantiser's decoded output (bfp16-exact bf16, blocks of 8 channels
// per pixel: the same blocks). Activations are row-major (H, W, C) bf16.
// When W % 128 == 0 (every VAE decoder stage) the GEMM reads its A tiles straight from the image: K step kt is 64
// channels of one tap, loaded per 128-pixel run by a 3-D TMA box at the tap's (dy, dx) offset, whose zero fill
// outside the image is the convolution's padding (implicit GEMM, no gather). Otherwise the activations are first
// gathered im2col-style into rows of the same K layout (zero outside the image and in the channel padding).
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace conv {

constexpr int kThreads = 256;

// The GEMM's K: taps^2 taps of C channels, each padded to the kernel's 64-deep K step (a K step never spans two
// taps; the bfp16 blocks of 8 channels of one tap are unchanged).
__host__ __device__ inline int64_t k_per_tap(int C) { return (static_cast<int64_t>(C) + 63) / 64 * 64; }
inline int64_t k_padded(int C, int taps) { return static_cast<int64_t>(taps) * taps * k_per_tap(C); }

// 0: the implicit GEMM where it applies, 1: always gather (rl_set_conv_path, for tests and benchmarks).
static int g_conv_path = 0;

// Gather: col[y * W + x][(dy * taps + dx) * Kt + c] = x[y + dy - taps / 2][x + dx - taps / 2][c] for c < C (0
// outside the image and for C <= c < Kt = k_per_tap(C)), in 16-byte groups of 8 channels; one thread per (pixel,
// 8-column group of Kp).
__global__ void __launch_bounds__(kThreads) im2col_kernel(const uint16_t* __restrict__ x, int H, int W, int C,
                                                          int taps, int64_t Kp, uint16_t* __restrict__ col) {
  const int groups = C >> 3;
  const int64_t kg = Kp >> 3, tg = k_per_tap(C) >> 3;   // 8-column groups per row / per tap
  const int64_t total = static_cast<int64_t>(H) * W * kg;
  const int half = taps >> 1;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t pix = i / kg, g8 = i % kg;
    uint4 v = make_uint4(0, 0, 0, 0);
    const int tap = static_cast<int>(g8 / tg), g = static_cast<int>(g8 % tg);
    if (g < groups) {
      const int y = static_cast<int>(pix / W), xx = static_cast<int>(pix % W);
      const int sy = y + tap / taps - half, sx = xx + tap % taps - half;
      if (sy >= 0 && sy < H && sx >= 0 && sx < W)
        v = __ldg(reinterpret_cast<const uint4*>(x + (static_cast<int64_t>(sy) * W + sx) * C) + g);
    }
    reinterpret_cast<uint4*>(col + pix * Kp)[g8] = v;
  }
}

// The input rows are already the GEMM's A rows for a 1x1 conv with C % 64 == 0; otherwise the implicit GEMM runs
// when the image allows it, and the gather when it does not.
inline bool direct(int C, int taps) { return taps == 1 && C % 64 == 0; }
inline bool implicit(int W, int C, int taps) { return !direct(C, taps) && g_conv_path == 0 && W % 128 == 0 && C >= 64; }
inline bool gathers(int W, int C, int taps) { return !direct(C, taps) && !implicit(W, C, taps); }

inline size_t workspace_bytes(int H, int W, int C, int taps) {
  return gathers(W, C, taps) ? static_cast<size_t>(H) * W * k_padded(C, taps) * 2 : 0;
}

}  // namespace conv
}  // namespace rl

extern "C" {

int rl_set_conv_path(int path) {
  const int prev = rl::conv::g_conv_path;
  rl::conv::g_conv_path = path;
  return prev;
}

size_t rl_conv2d_workspace(int H, int W, int Cin, int taps) {
  if (H <= 0 || W <= 0 || Cin <= 0 || (taps != 1 && taps != 3)) return 0;
  return rl::conv::workspace_bytes(H, W, Cin, taps);
}

int rl_conv2d_bfp16(const uint16_t* x, int H, int W, int Cin, const uint8_t* w_native, int Cout, int taps,
                    const uint16_t* bias, uint16_t* out, void* workspace, size_t workspace_bytes,
                    rl_stream_t stream) {
  using namespace rl;
  RL_REQUIRE(x && w_native && out, RL_ERR_ARGUMENT, "rl_conv2d_bfp16: NULL pointer");
  RL_REQUIRE(H > 0 && W > 0 && (taps == 1 || taps == 3), RL_ERR_ARGUMENT, "rl_conv2d_bfp16: need H, W > 0, taps 1/3");
  RL_REQUIRE(Cin > 0 && Cin % 8 == 0 && Cout > 0 && Cout % 128 == 0, RL_ERR_ARGUMENT,
             "rl_conv2d_bfp16: need Cin %% 8 == 0 and Cout %% 128 == 0 (Cin=%d Cout=%d)", Cin, Cout);
  const size_t need = conv::workspace_bytes(H, W, Cin, taps);
  RL_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr), RL_ERR_ARGUMENT,
             "rl_conv2d_bfp16: workspace of %zu bytes, need %zu", workspace_bytes, need);
  RL_REQUIRE(aligned(x, 16) && aligned(workspace, 16), RL_ERR_ALIGNMENT, "rl_conv2d_bfp16: 16-byte alignment");
  const int64_t M = static_cast<int64_t>(H) * W;
  const int64_t Kp = conv::k_padded(Cin, taps);
  if (conv::implicit(W, Cin, taps)) {
    RL_REQUIRE(w_native && aligned(w_native, 16) && aligned(out, 16), RL_ERR_ALIGNMENT,
               "rl_conv2d_bfp16: 16-byte alignment");
    RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_conv2d_bfp16: needs an sm_100 device");
    return gemm::linear_conv(x, H, W, Cin, taps, w_native, Cout, bias, out, stream);
  }
  const uint16_t* a = x;
  if (conv::gathers(W, Cin, taps)) {
    RL_REQUIRE(device_is_sm100(), RL_ERR_UNSUPPORTED, "rl_conv2d_bfp16: needs an sm_100 device");
    uint16_t* col = static_cast<uint16_t*>(workspace);
    const int64_t work = M * (Kp / 8);
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    const int64_t blocks = (work + conv::kThreads - 1) / conv::kThreads;
    conv::im2col_kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), conv::kThreads, 0, stream>>>(
        x, H, W, Cin, taps, Kp, col);
    RL_TRY_CUDA(cudaGetLastError());
    a = col;
  }
  return rl_linear_bfp16(a, M, Kp, w_native, Cout, bias, bias ? RL_EPI_BIAS : RL_EPI_NONE, out, RL_BF16, stream);
}

}  // extern "C"
