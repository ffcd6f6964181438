"""ctypes binding of libredline_b200.so (the C ABI declared in include/redline_b200.h).

The library is built in-tree by `redline_tiny_b200.build` (nvcc, sm_100a). There is no CPU fallback: if the
library is missing or the device is not an sm_100 GPU, calls raise RedlineError.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libredline_b200.so")

RL_OK, RL_ERR_ARGUMENT, RL_ERR_ALIGNMENT, RL_ERR_UNSUPPORTED, RL_ERR_CUDA, RL_ERR_DEVICE = 0, -1, -2, -3, -4, -5
RL_F32, RL_BF16 = 0, 1
RL_ROWMAJOR, RL_A_LAYOUT, RL_C_ATB = 0, 1, 2
RL_EPI_NONE, RL_EPI_BIAS, RL_EPI_SWIGLU = 0, 1, 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (restype, argtypes); mirrors include/redline_b200.h
SIGNATURES = {
    "rl_last_error": (ctypes.c_char_p, []),
    "rl_version": (_I, []),
    "rl_device_status": (_I, [ctypes.POINTER(_I)]),
    "rl_quantize_bfp16": (_I, [_P, _I, _I64, _I64, _I, _P, _P, _P]),
    "rl_dequantize_bfp16": (_I, [_P, _I, _I64, _I64, _P, _I, _P]),
    "rl_pack_b": (_I, [_P, _I, _I64, _I64, _P, _P]),
    "rl_permute_bf16": (_I, [_P, _I, _P, _I, _I64, _I64, _P]),
    "rl_weights_from_pack_b": (_I, [_P, _I64, _I64, _I, _P, _P]),
    "rl_pack_weights": (_I, [_P, _I, _I64, _I64, _I, _P, _P]),
    "rl_weights_shard": (_I, [_I64, _I64, _I, _I, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                              ctypes.POINTER(_I64)]),
    "rl_linear_bfp16": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _P, _I, _P]),
    "rl_linear_bfp16_workspace": (ctypes.c_size_t, [_I64, _I64, _I64, _I]),
    "rl_linear_bfp16_ws": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _P, _I, _P, ctypes.c_size_t, _P]),
    "rl_set_gemm_variant": (_I, [_I]),
    "rl_gemm_pair_clusters": (_I, []),
    "rl_set_attention_variant": (_I, [_I]),
    "rl_set_conv_path": (_I, [_I]),
    "rl_conv2d_workspace": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "rl_conv2d_bfp16": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _P, _P, ctypes.c_size_t, _P]),
    "rl_swiglu_mlp_workspace": (ctypes.c_size_t, [_I64, _I64, _I64, _I]),
    "rl_attention": (_I, [_P, _P, _P, _I64, _I, _I64, _I64, _I64, _P, ctypes.c_float, _P, _I64, _P]),
    "rl_swiglu_mlp_noalloc_capacity": (ctypes.c_size_t, []),
    "rl_swiglu_mlp_noalloc": (_I, [_P, _I, _I, _I64, _I64, _P, _I64, _P, _I64, _P, _I, _P]),
    "rl_ln_mod": (_I, [_P, _P, _I, _P, _I64, _I64, _I64, _P, _P, _P, _P]),
    "rl_qkv_post": (_I, [_P, _P, _P, _P, _I64, _I, _P, _P, _P, _I64, _P]),
    "rl_qkv_post_gqa": (_I, [_P, _P, _P, _P, _I64, _I, _I, _P, _P, _P, _I64, _P]),
    "rl_qkv_linear": (_I, [_P, _I64, _I64, _P, _I, _I, _P, _P, _P, _P, _P, _P, _I64, _P]),
    "rl_rms_mod": (_I, [_P, _P, _I, _P, _I64, _I64, _I64, _P, _P, _P, _P]),
    "rl_attention_gqa": (_I, [_P, _P, _P, _I64, _I, _I, _I64, _I64, _I64, _P, ctypes.c_float, _P, _I64, _P]),
    "rl_attention_gqa_f32": (_I, [_P, _P, _P, _I64, _I, _I, _I64, _I64, _I64, _P, ctypes.c_float, _P, _I64, _P]),
    "rl_swiglu_mlp": (_I, [_P, _I, _I, _I64, _I64, _P, _I64, _P, _I64, _P, _I, _P, ctypes.c_size_t, _P]),
    "rl_matvec_f32": (_I, [_P, _I, _I, _P, _I, _P, _I, _P, _P]),
    "rl_sinusoidal_embed": (_I, [ctypes.c_float, ctypes.c_float, _P, _I, _P, _P]),
    "rl_adaln_params": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "rl_npu_qkv_pack": (_I, [_P, _P, _P, _I64, _I, _I, _P, _P, _P]),
    "rl_npu_q_unpack": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "rl_npu_kv_unpack": (_I, [_P, _I, _I, _I, _I, _I64, _I64, _I64, _P, _P, _P]),
    "rl_npu_qkv_tables": (_I, [_P, _I, _P, _P, _P, _P]),
    "rl_linear_bfp16_mirror": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _P, _P, _I, _P]),
    "rl_linear_bfp16_partial": (_I, [_P, _I64, _I64, _P, _I64, _P, _P, _P]),
    "rl_linear_bfp16_scatter": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _I64, _P]),
    "rl_ln_mod_tp_rs": (_I, [_P, _P, _I, _P, _I, ctypes.c_ulonglong, _P, _I64, _I64, _I64, _P, _P, _P]),
    "rl_tp_wait": (_I, [_P, _I, _I, ctypes.c_ulonglong, _P]),
    "rl_ipc_alloc": (_I, [_I64, _P, _P]),
    "rl_ipc_open": (_I, [_P, _P]),
    "rl_ipc_close": (_I, [_P]),
    "rl_ipc_free": (_I, [_P]),
    "rl_tp_signal": (_I, [_P, _I, _I, _I, ctypes.c_ulonglong, _P]),
    "rl_ln_mod_tp": (_I, [_P, _P, _I, _P, _I, ctypes.c_ulonglong, _P, _I64, _I64, _I64, _P, _P, _P, _P]),
}


class RedlineError(RuntimeError):
    """A C-ABI call returned an error status (message from rl_last_error)."""

    def __init__(self, fn, status, msg):
        super().__init__(f"{fn} failed ({status}): {msg}")
        self.status = status


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RedlineError("load", RL_ERR_UNSUPPORTED,
                               f"{LIB_PATH} is not built; run `python -m redline_tiny_b200.build`")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype, f.argtypes = res, args
        _lib = h
    return _lib


def call(name, *args):
    """Call a C-ABI entry point; raise RedlineError on a non-zero status."""
    st = getattr(lib(), name)(*args)
    if st != RL_OK:
        raise RedlineError(name, st, lib().rl_last_error().decode(errors="replace"))
    return st


def device_status():
    """Synchronise and read / clear the device error word; raises on a device-side error."""
    flags = ctypes.c_int(0)
    st = lib().rl_device_status(ctypes.byref(flags))
    if st != RL_OK:
        raise RedlineError("rl_device_status", st, lib().rl_last_error().decode(errors="replace"))
    return flags.value
