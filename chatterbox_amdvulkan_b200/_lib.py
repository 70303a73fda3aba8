"""ctypes binding of libcbx_ops.so (the C ABI declared in include/cbx_ops.h).

The library is built in-tree by ``chatterbox_amdvulkan_b200.build``.  There is
no fallback: if the shared object is missing or cannot be loaded, every op
raises instead of computing anything on the CPU.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
# CBX_LIB_PATH selects another build of the same ABI (A/B measurements).
LIB_PATH = os.environ.get("CBX_LIB_PATH") or os.path.join(PKG, "libcbx_ops.so")

# cbx_type (numerically ggml_type)
F32, F16, BF16 = 0, 1, 30
# cbx_layout
BCT, BTC = 0, 1
# cbx_act
ACT_NONE, ACT_MISH, ACT_SILU, ACT_GELU_TANH = 0, 1, 2, 3
ACT_GELU_ERF, ACT_LEAKY_RELU, ACT_ELU = 4, 5, 6
# cbx_bias_axis
BIAS_NE0, BIAS_NE1 = 0, 1
# error-word bits of cbx_embed_gather_add
EFLAG_TOKEN_OOB, EFLAG_POS_OOB = 0x1, 0x2
# bits of the library's device error word (cbx_device_errors)
DEVERR_WAIT_TIMEOUT = 0x1

STATUS = {0: "CBX_OK", -1: "CBX_ERR_INVALID_ARG", -2: "CBX_ERR_UNSUPPORTED_DTYPE",
          -3: "CBX_ERR_LAUNCH", -4: "CBX_ERR_INDEX_OOB", -5: "CBX_ERR_TIMEOUT",
          -6: "CBX_ERR_CUDA"}

# Every symbol include/cbx_ops.h declares, with its ctypes signature.
_vp, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "cbx_version": ([], ctypes.c_int),
    "cbx_last_error": ([], ctypes.c_char_p),
    "cbx_status_string": ([_i32], ctypes.c_char_p),
    "cbx_device_errors": ([_vp, _vp], ctypes.c_int),
    "cbx_selftest_wait_timeout": ([ctypes.c_uint32, _vp], ctypes.c_int),
    "cbx_embed_gather_add": ([_vp, _i32, _i64, _vp, _i32, _i64, _vp, _vp, _i64, _i64, _i64, _vp,
                              _i32, _vp, _vp], ctypes.c_int),
    "cbx_embed_gather_add_batched": ([_vp, _i32, _i64, _vp, _i32, _i64, _vp, _i64, _i64, _i64,
                                      _i64, _vp, _i32, _vp, _vp], ctypes.c_int),
    "cbx_t3_embed_sequence": ([_vp, _i64, _vp, _i32, _i64, _vp, _i64, _vp, _i32, _i64, _vp, _i64,
                               _vp, _i32, _i64, _i64, _i64, _vp, _i32, _vp, _vp], ctypes.c_int),
    "cbx_t3_embed_sequence_batched": ([_vp, _i64, _vp, _i32, _i64, _vp, _i64, _vp, _i32, _i64,
                                       _vp, _i64, _vp, _i32, _i64, _i64, _i64, _i64, _vp, _i32,
                                       _vp, _vp], ctypes.c_int),
    "cbx_add_layernorm": ([_vp, _vp, _i32, _i64, _vp, _vp, _f32, _i64, _i64, _vp, _vp, _i32, _i64,
                           _vp], ctypes.c_int),
    "cbx_layernorm_channels": ([_vp, _vp, _vp, _f32, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _vp],
                               ctypes.c_int),
    "cbx_causal_block1d_tail": ([_vp, _vp, _vp, _vp, _f32, _vp, _i64, _i64, _i64, _i32, _vp,
                                 _vp], ctypes.c_int),
    "cbx_gelu_tanh": ([_vp, _vp, _i64, _i32, _vp], ctypes.c_int),
    "cbx_silu": ([_vp, _vp, _i64, _i32, _vp], ctypes.c_int),
    "cbx_mish": ([_vp, _vp, _i64, _i32, _vp], ctypes.c_int),
    "cbx_gelu_erf": ([_vp, _vp, _i64, _i32, _vp], ctypes.c_int),
    "cbx_bias_act": ([_vp, _vp, _i32, _i64, _i64, _vp, _i32, _i64, _i32, _f32, _vp], ctypes.c_int),
    "cbx_sum3_scale": ([_vp, _vp, _vp, _f32, _vp, _i64, _i32, _vp], ctypes.c_int),
    "cbx_timestep_embed": ([_vp, _i64, _vp, _i32, _f32, _i32, _vp, _vp], ctypes.c_int),
    "cbx_sinusoid_freqs": ([_i32, _vp], ctypes.c_int),
    "cbx_snake": ([_vp, _vp, _vp, _f32, _i64, _i64, _i64, _i32, _vp, _vp], ctypes.c_int),
    "cbx_snake_alpha_inv": ([_vp, _i64, _f32, _vp], ctypes.c_int),
    "cbx_nsf_source": ([_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _f32, _vp, _vp], ctypes.c_int),
    "cbx_stft": ([_vp, _i64, _i64, _i32, _i32, _vp, _i32, _vp, _vp], ctypes.c_int),
    "cbx_istft_post": ([_vp, _i64, _i64, _i32, _i32, _vp, _i32, _f32, _vp, _vp], ctypes.c_int),
    "cbx_hann_window": ([_i32, _vp], ctypes.c_int),
    "cbx_qkv_kv_append": ([_vp, _i64, _vp, _i64, _i64, _vp, _i32, _vp, _vp, _i32, _i64, _i64, _vp,
                           _vp, _vp], ctypes.c_int),
}

_lock = threading.Lock()
_lib = None


class CbxError(RuntimeError):
    """A libcbx_ops call returned a negative status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn}: {STATUS.get(status, status)}: {msg}")
        self.status = status


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libcbx_ops.so (once) and attach the signatures of include/cbx_ops.h."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libcbx_ops.so not found at {path}; build it with "
                    "`python -m chatterbox_amdvulkan_b200.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(path)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def check(fn: str, status: int) -> None:
    if status != 0:
        msg = load().cbx_last_error()
        raise CbxError(fn, status, msg.decode() if msg else "")


def call(fn: str, *args) -> None:
    """Call a cbx_* entry point and raise CbxError on a negative status."""
    check(fn, getattr(load(), fn)(*args))
