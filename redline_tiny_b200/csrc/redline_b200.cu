// Single translation unit of libredline_b200.so: the kernels share one device error word (rl::g_device_error), so
// every part is compiled together rather than linked with relocatable device code.
#include "rl_capi.cu"
#include "rl_codec.cu"
#include "rl_gemm.cu"
#include "rl_glue.cu"
#include "rl_attn.cu"
#include "rl_conv.cu"
#include "rl_adaln.cu"
#include "rl_npu.cu"
#include "rl_tp.cu"
