// VAE decoder convolution (3x3 pad 1, or 1x1; stride 1) with bfp16 weights, as a GEMM on the packed-weight kernel.
//
// Restates the reference's vconv (kernels/vae/vconv.cc:1-17, weights packed by redline/vae_ops.py:44-61
// pack_vconv, checked against vae_ops.conv_ref, vae_ops.py:64-75): out[y][x][co] = b[co] +
// sum_{dy,dx,ci} in[y+dy-1][x+dx-1][ci] * w[co][ci][dy][dx]. The reference quantises its weights to bfp16 blocks of
// 8 input channels per (output channel, tap) and its activation strips to bfp16 blocks of 8 channels per pixel; here
// the weights are the GEMM's B = [(dy, dx, ci)][co] in the native tile format (blocks of 8 along K = 8 input
// channels of one tap: the same blocks), and the activations are the quantiser's decoded output (bfp16-exact bf16,
// blocks of 8 channels per pixel: the same blocks), gathered im2col-style into rows of K = taps^2 * Cin (zero outside
// the image), padded with zero columns to a multiple of 64, and multiplied by rl_linear_bfp16 with the bias epilogue.
// Activations are row-major (H, W, C) bf16.
#include "rl_common.cuh"
#include "rl_host.h"

namespace rl {
namespace conv {

constexpr int kThreads = 256;

// The GEMM's K: taps^2 * C rounded up to the kernel's 64-deep K step (zero columns after the last tap, so the
// bfp16 blocks of 8 channels of one tap are unchanged).
inline int64_t k_padded(int C, int taps) { return (static_cast<int64_t>(taps) * taps * C + 63) / 64 * 64; }

// Gather: col[y * W + x][(dy * taps + dx) * C + c] = x[y + dy - taps / 2][x + dx - taps / 2][c] (0 outside the image
// and in the pad columns up to Kp), in 16-byte groups of 8 channels; one thread per (pixel, 8-column group of Kp).
__global__ void __launch_bounds__(kThreads) im2col_kernel(const uint16_t* __restrict__ x, int H, int W, int C,
                                                          int taps, int64_t Kp, uint16_t* __restrict__ col) {
  const int groups = C >> 3;
  const int64_t kg = Kp >> 3, real = static_cast<int64_t>(taps) * taps * groups;
  const int64_t total = static_cast<int64_t>(H) * W * kg;
  const int half = taps >> 1;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t pix = i / kg, g8 = i % kg;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (g8 < real) {
      const int tap = static_cast<int>(g8 / groups), g = static_cast<int>(g8 % groups);
      const int y = static_cast<int>(pix / W), xx = static_cast<int>(pix % W);
      const int sy = y + tap / taps - half, sx = xx + tap % taps - half;
      if (sy >= 0 && sy < H && sx >= 0 && sx < W)
        v = __ldg(reinterpret_cast<const uint4*>(x + (static_cast<int64_t>(sy) * W + sx) * C) + g);
    }
    reinterpret_cast<uint4*>(col + pix * Kp)[g8] = v;
  }
}

// The gather is needed unless the input rows are already the GEMM's A rows (a 1x1 conv with C % 64 == 0).
inline bool gathers(int C, int taps) { return taps != 1 || C % 64 != 0; }

inline size_t workspace_bytes(int H, int W, int C, int taps) {
  return gathers(C, taps) ? static_cast<size_t>(H) * W * k_padded(C, taps) * 2 : 0;
}

}  // namespace conv
}  // namespace rl

extern "C" {

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
  const uint16_t* a = x;
  if (conv::gathers(Cin, taps)) {
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
