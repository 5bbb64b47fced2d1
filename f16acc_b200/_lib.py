"""Loader for the native library libf16acc_b200.so (the C ABI of include/f16acc.h).

The library must have been built (``python -m f16acc_b200.build`` or the repo's
``__graft_entry__.build()``); there is no fallback implementation, so a missing
or unloadable library raises at first use.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libf16acc_b200.so")

# Every symbol include/f16acc.h declares, with its ctypes signature.
_i64 = ctypes.c_int64
_int = ctypes.c_int
_p = ctypes.c_void_p
_size = ctypes.c_size_t


class Plan(ctypes.Structure):
    _fields_ = [("variant", ctypes.c_int), ("tile_m", ctypes.c_int), ("tile_n", ctypes.c_int),
                ("tiles_m", ctypes.c_int64), ("tiles_n", ctypes.c_int64)]


_GEMM_ARGS = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _int, _i64, _i64, _i64, _int, _p, _size, _int, _p]

SIGNATURES = {
    "f16acc_gemm": (_int, _GEMM_ARGS),
    "f16acc_gemm_ex": (_int, _GEMM_ARGS + [_int]),
    "f16acc_gemm_main": (_int, _GEMM_ARGS + [_int]),
    "f16acc_gemm_redo": (_int, _GEMM_ARGS + [_int]),
    "f16acc_gemm_bias": (_int, _GEMM_ARGS[:6] + [_p, _i64] + _GEMM_ARGS[6:] + [_int]),
    "f16acc_gemm_allgather": (_int, [_p, _i64, _i64, _p, _i64, _i64, ctypes.POINTER(ctypes.c_void_p), _int, _i64, _i64,
                                     _int, _i64, _i64, _i64, _int, _p, _size, _int, _p]),
    "f16acc_workspace_bytes": (_size, [_i64, _i64, _i64]),
    "f16acc_strerror": (ctypes.c_char_p, [_int]),
    "f16acc_get_plan": (_int, [_p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _int, ctypes.POINTER(Plan)]),
    "f16acc_flag_bytes_per_tile": (_int, []),
    "f16acc_set_tc_config": (_int, [_int, _int]),
    "f16acc_set_sm_limit": (_int, [_int]),
    "f16acc_set_redo_mode": (_int, [_int]),
    "f16acc_set_schedule": (_int, [_int]),
    "f16acc_set_fp32_tiles": (_int, [_int]),
    "f16acc_set_tail_split": (_int, [_int]),
    "f16acc_probe_chunk_rate": (_int, [_int, _int, _int, _int, _p, _int, _p]),
    "f16acc_selftest_wait_timeout": (_int, [ctypes.c_uint64, _p, _int, _p]),
    "f16acc_device_status": (_int, [_int, _int]),
    "f16acc_gemm_noalloc": (_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _int, _i64, _i64, _i64, _int,
                                   _int, _p]),
    "f16acc_version": (ctypes.c_char_p, []),
}

# Return codes and constants (include/f16acc.h).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_WORKSPACE = 2
ERR_UNSUPPORTED = 3
ERR_CUDA = 4
ERR_DEVICE_TIMEOUT = 5
ERR_TOO_LARGE = 6
NOALLOC_MAX_TILES = 65536
OUT_F16, OUT_F32, OUT_BF16 = 0, 1, 2
VARIANT_AUTO, VARIANT_TCGEN05, VARIANT_MMA_SYNC, VARIANT_SKINNY = 0, 1, 2, 3
VARIANT_NAMES = {VARIANT_AUTO: "auto", VARIANT_TCGEN05: "tcgen05", VARIANT_MMA_SYNC: "mma_sync",
                 VARIANT_SKINNY: "skinny"}
REDO_SEPARATE, REDO_INLINE = 0, 1
SCHEDULE_STATIC, SCHEDULE_DYNAMIC = 0, 1
FP32_TILES_AUTO, FP32_TILES_WIDE, FP32_TILES_NARROW = 0, 1, 2
TAIL_SPLIT_OFF, TAIL_SPLIT_ON = 0, 1

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """The loaded library with argtypes set; raises RuntimeError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"f16acc_b200 native library missing at {LIB_PATH}; "
                                   "build it with `python -m f16acc_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().f16acc_strerror(code).decode()
