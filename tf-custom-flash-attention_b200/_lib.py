"""ctypes binding of libsdpa_b200.so (the C ABI of include/sdpa_b200.h).

The library is required: importing this module on a machine where it has not
been built raises, and there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsdpa_b200.so")

OK, EINVAL, EUNSUPPORTED, ECUDA, ETIMEOUT, EWORKSPACE, ESCRATCH = range(7)
NOALLOC_MAX_ROWS = 1 << 20
F16, F32 = 0, 1

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run tf-custom-flash-attention_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, u64, f32, ci, sz = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_int,
                                 ctypes.c_size_t)
    L.sdpa_b200_fwd.argtypes = [ci, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, f32, ci, u64, u64, vp]
    L.sdpa_b200_fwd.restype = ci
    L.sdpa_b200_bwd_workspace_bytes.argtypes = [ci, i64, i64, i64, i64, i64]
    L.sdpa_b200_bwd_workspace_bytes.restype = sz
    L.sdpa_b200_bwd.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, f32, ci, u64,
                                u64, vp, sz, vp]
    L.sdpa_b200_bwd.restype = ci
    L.sdpa_b200_bwd_dstats.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, f32,
                                       ci, u64, u64, vp, sz, vp]
    L.sdpa_b200_bwd_dstats.restype = ci
    L.sdpa_b200_bwd_noalloc.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, f32,
                                        ci, u64, u64, vp]
    L.sdpa_b200_bwd_noalloc.restype = ci
    L.sdpa_b200_fwd_bshd.argtypes = [ci, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, f32, f32, ci, u64, u64,
                                     vp]
    L.sdpa_b200_fwd_bshd.restype = ci
    L.sdpa_b200_bwd_bshd.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, f32,
                                     f32, ci, u64, u64, vp, sz, vp]
    L.sdpa_b200_bwd_bshd.restype = ci
    L.sdpa_b200_last_error_detail.argtypes = []
    L.sdpa_b200_last_error_detail.restype = ctypes.c_char_p
    L.sdpa_b200_dropout_mask.argtypes = [u64, u64, i64, i64, i64, f32, vp, vp]
    L.sdpa_b200_dropout_mask.restype = ci
    L.sdpa_b200_strerror.argtypes = [ci]
    L.sdpa_b200_strerror.restype = ctypes.c_char_p
    L.sdpa_b200_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint), vp]
    L.sdpa_b200_device_status.restype = ci
    L.sdpa_b200_set_wait_timeout_ns.argtypes = [u64]
    L.sdpa_b200_set_wait_timeout_ns.restype = None
    L.sdpa_b200_test_wait_timeout.argtypes = [u64, vp]
    L.sdpa_b200_test_wait_timeout.restype = ci
    L.sdpa_b200_path.argtypes = [ci, i64, i64, ci]
    L.sdpa_b200_path.restype = ci
    L.sdpa_b200_last_launch_count.restype = ci
    L.sdpa_b200_version.restype = ci
    L.sdpa_b200_set_bwd_events.argtypes = [vp, ci]
    L.sdpa_b200_set_bwd_events.restype = ci
    _lib = L
    return L


def strerror(code: int) -> str:
    return lib().sdpa_b200_strerror(code).decode()


# Every symbol include/sdpa_b200.h declares (checked by the CPU tests).
EXPORTS = (
    "sdpa_b200_fwd", "sdpa_b200_bwd_workspace_bytes", "sdpa_b200_bwd", "sdpa_b200_dropout_mask",
    "sdpa_b200_strerror", "sdpa_b200_device_status", "sdpa_b200_set_wait_timeout_ns",
    "sdpa_b200_test_wait_timeout", "sdpa_b200_path", "sdpa_b200_last_launch_count", "sdpa_b200_version",
    "sdpa_b200_bwd_noalloc", "sdpa_b200_bwd_dstats", "sdpa_b200_set_bwd_events", "sdpa_b200_fwd_bshd",
    "sdpa_b200_bwd_bshd", "sdpa_b200_last_error_detail",
)
