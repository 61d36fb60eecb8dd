"""ctypes binding of libtau_dxb.so (the C ABI declared in include/tau_dxb.h).

The library is built in-tree by tau_dxb_b200/build.py. Loading fails loudly
when it is missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libtau_dxb.so")

# status codes / enums (mirror include/tau_dxb.h)
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_WORKSPACE = -4
ERR_NO_DEVICE = -5

F32, BF16, F16 = 0, 1, 2
SIGMA_IDS = {"softplus": 0, "sigmoid": 1, "exp": 2, "relu": 3}
FIXED_SIGMA_IDS = dict(SIGMA_IDS, tanh_shift=4)      # the fixed-tau weights add tanh_shift
PATH_AUTO, PATH_PRECISE, PATH_TENSOR = 0, 1, 2
WTA_THRESHOLD, WTA_EXACT_K = 0, 1
WTA_GELU_INPUT = 0x100
TAU_STAR_MAX_KEYS = 28672
DEVERR_SELFTEST = 0x100

_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64

# name -> (restype, argtypes); every function include/tau_dxb.h declares
SIGNATURES = {
    "tau_dxb_version": (ctypes.c_int, []),
    "tau_dxb_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "tau_dxb_last_error": (ctypes.c_char_p, []),
    "tau_dxb_device_error": (ctypes.c_int, [ctypes.c_int32]),
    "tau_dxb_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_int32), _vp]),
    "tau_attn_fwd": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p,           # q, k, v
        _i32, _i64, _i64, _i64, _i64, _i64,           # dtype, B, H, Lq, Lk, D
        _vp, _vp, _i32, ctypes.c_float,               # tau, alpha, sigma, scale
        _vp, _i32, _i64p, _i32,                       # mask, mask dtype, strides, causal
        _vp, _i64p,                                   # out
        _vp, _vp, _vp,                                # row_max, row_z, row_argmax
        _i32, _vp]),                                  # path, stream
    "tau_attn_bwd_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64]),
    "whisper_log_mel_workspace_bytes": (ctypes.c_size_t, [_i64]),
    "whisper_log_mel": (ctypes.c_int, [_vp, _i64, _i64, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "tau_attn_bwd": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p,           # q, k, v
        _vp, _i64p, _vp, _i64p,                       # out, dout
        _i32, _i64, _i64, _i64, _i64, _i64,           # dtype, B, H, Lq, Lk, D
        _vp, _vp, _i32, ctypes.c_float,               # tau, alpha, sigma, scale
        _vp, _i32, _i64p, _i32,                       # mask
        _vp, _vp, _vp,                                # row state
        _vp, _i64p, _vp, _i64p, _vp, _i64p,           # dq, dk, dv
        _vp, _vp,                                     # dtau, dalpha
        _vp, ctypes.c_size_t,                         # workspace
        _i32, _vp]),                                  # path, stream
    "tau_attn_bwd_noalloc": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p,           # q, k, v
        _vp, _i64p, _vp, _i64p,                       # out, dout
        _i32, _i64, _i64, _i64, _i64, _i64,           # dtype, B, H, Lq, Lk, D
        _vp, _vp, _i32, ctypes.c_float,               # tau, alpha, sigma, scale
        _vp, _i32, _i64p, _i32,                       # mask
        _vp, _vp, _vp,                                # row state
        _vp, _i64p, _vp, _i64p, _vp, _i64p,           # dq, dk, dv
        _vp, _vp,                                     # dtau, dalpha
        _i32, _vp]),                                  # path, stream
    "wta_fwd": (ctypes.c_int, [_vp, _i32, _i64, _i64, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _vp]),
    "wta_bwd": (ctypes.c_int, [_vp, _i32, _vp, _i64, _i64, _vp, _vp]),
    "wta_bwd_gelu": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp]),
    "wta_k_from_logits": (ctypes.c_int, [_vp, _i64, _i64, _vp, _vp]),
    "tau_star_solve": (ctypes.c_int, [_vp, _i64, _i64, _i64, _i32, _i32, ctypes.c_float, ctypes.c_float,
                                      ctypes.c_float, ctypes.c_float, _vp, _vp, _vp]),
    "tau_star_analytic": (ctypes.c_int, [_vp, _i64, _i64, _i64, _i32, _vp, _vp]),
    "tau_layer_norm_fwd": (ctypes.c_int, [_vp, _i64, _i64, _vp, _vp, ctypes.c_float, _vp, _i32, _vp, _vp, _vp]),
    "tau_layer_norm_bwd_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "tau_layer_norm_bwd": (ctypes.c_int, [_vp, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp,
                                          ctypes.c_size_t, _vp]),
    "tau_column_sum_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "tau_column_sum": (ctypes.c_int, [_vp, _i32, _i64, _i64, _vp, _i32, _vp, ctypes.c_size_t, _vp]),
    "tau_grad_mask": (ctypes.c_int, [_vp, _i32, _i64, _i64, _vp, _i32, _vp, _vp]),
    "tau_opus_fixed_fwd": (ctypes.c_int, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i32, _vp, _vp]),
    "tau_opus_fixed_bwd": (ctypes.c_int, [_vp, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i32, _vp, _vp]),
    "tau_cross_entropy_fwd": (ctypes.c_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "tau_cross_entropy_bwd": (ctypes.c_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp]),
}

_lib = None
_lock = threading.Lock()


class TauDxbError(RuntimeError):
    """A libtau_dxb entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str):
        self.status = status
        super().__init__(f"{fn} failed ({status}: {strerror(status)}): {detail}")


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"tau_dxb_b200: CUDA library not built ({LIB_PATH} missing); "
                    "run `python -m tau_dxb_b200.build` (nvcc, sm_100a)")
            handle = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def strerror(status: int) -> str:
    return lib().tau_dxb_strerror(status).decode()


def last_error() -> str:
    return lib().tau_dxb_last_error().decode()


def check(fn_name: str, status: int) -> None:
    if status != OK:
        raise TauDxbError(fn_name, status, last_error())


def strides4(t) -> ctypes.Array:
    s = list(t.stride())
    assert len(s) == 4
    return (ctypes.c_int64 * 4)(*s)


NULL4 = None


def dtype_code(dt) -> int:
    import torch
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise TypeError(f"tau_dxb_b200: unsupported dtype {dt} (float32, bfloat16, float16)")


def stream_ptr(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
