"""ctypes front end of the CPU oracle (oracle/f16acc_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by `__graft_entry__.smoke()` and
by bench.py's CPU-baseline leg, as the checker.  The product package
(f16acc_b200) never imports it and has no CPU fallback.

All functions take numpy float16 arrays with any element strides (views,
transposes) and hand them to C without copying.  Reference semantics cited in
the C file header (steppergg/f16acc f16acc/kernel.py:37-81).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_f16acc.so")
_lib = None

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


def build() -> str:
    """Compile the oracle with the committed Makefile (gcc + OpenMP)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_gemm_f64.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64]
        L.oracle_gemm_f32acc.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64]
        L.oracle_gemm_chunked.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64,
                                          ctypes.c_int, ctypes.c_int, _i64, _i64, _p, ctypes.c_int]
        L.oracle_gemm_chunked_rows.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64,
                                               ctypes.c_int, ctypes.c_int, _i64, _i64]
        L.oracle_round_f16.argtypes = [_p, _p, _i64]
        L.oracle_rel.argtypes = [_p, _p, _i64]
        L.oracle_rel.restype = ctypes.c_double
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _operand(x: np.ndarray):
    if x.dtype != np.float16 or x.ndim != 2:
        raise ValueError("oracle operands are 2-D float16 arrays")
    s0, s1 = (s // 2 for s in x.strides)
    if any(s % 2 for s in x.strides):
        raise ValueError("strides must be whole elements")
    return x.ctypes.data, s0, s1


def _check(a, b):
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"(M, K) @ (K, N) needed, got {a.shape} @ {b.shape}")


def gemm_f64(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """FP64 product a @ b (the accuracy reference, tests/test_f16acc.py:22-29)."""
    _check(a, b)
    (pa, a0, a1), (pb, b0, b1) = _operand(a), _operand(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), dtype=np.float64)
    lib().oracle_gemm_f64(pa, a0, a1, pb, b0, b1, c.ctypes.data, M, N, K)
    return c


def gemm_f32acc(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """FP32-accumulate product (kernel.py:50-51, the `chunked=False` mode)."""
    _check(a, b)
    (pa, a0, a1), (pb, b0, b1) = _operand(a), _operand(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), dtype=np.float32)
    lib().oracle_gemm_f32acc(pa, a0, a1, pb, b0, b1, c.ctypes.data, M, N, K)
    return c


def gemm_chunked(a: np.ndarray, b: np.ndarray, *, chunk: int = 32, round_every: int = 32,
                 tile: tuple[int, int] | None = None, redo: bool = True):
    """Chunked FP16-accumulate product, FP32 result before the final cast.

    With `tile=(bm, bn)` the per-tile overflow flags are computed (kernel.py:70-71)
    and, when `redo`, flagged tiles are replaced by the FP32-accumulate product
    (kernel.py:75-81).  Returns (c, flags) where flags is None without `tile`,
    else a uint8 array [cdiv(M,bm), cdiv(N,bn)].
    """
    _check(a, b)
    (pa, a0, a1), (pb, b0, b1) = _operand(a), _operand(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), dtype=np.float32)
    flags = None
    bm = bn = 0
    pflags = None
    if tile is not None:
        bm, bn = tile
        flags = np.zeros(((M + bm - 1) // bm, (N + bn - 1) // bn), dtype=np.uint8)
        pflags = flags.ctypes.data
    lib().oracle_gemm_chunked(pa, a0, a1, pb, b0, b1, c.ctypes.data, M, N, K,
                              chunk, round_every, bm, bn, pflags, 1 if redo else 0)
    return c, flags


def gemm_chunked_rows(a: np.ndarray, b: np.ndarray, row0: int, row1: int, *, round_every: int = 32):
    """Chunked product of rows [row0, row1) only (a bounded timing sample)."""
    _check(a, b)
    (pa, a0, a1), (pb, b0, b1) = _operand(a), _operand(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.zeros((M, N), dtype=np.float32) if M * N <= (1 << 26) else np.empty((M, N), dtype=np.float32)
    lib().oracle_gemm_chunked_rows(pa, a0, a1, pb, b0, b1, c.ctypes.data, M, N, K, 32, round_every, row0, row1)
    return c


def round_f16(x: np.ndarray) -> np.ndarray:
    """FP32 -> FP16 round-to-nearest-even (the fp16 store of kernel.py:59)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.float16)
    lib().oracle_round_f16(x.ctypes.data, out.ctypes.data, x.size)
    return out


def set_threads(n: int) -> int:
    """Use n OpenMP threads (e.g. os.cpu_count() under a launcher that pinned
    OMP_NUM_THREADS=1); returns the count now in effect."""
    lib().oracle_set_threads(int(n))
    return int(lib().oracle_threads())


def threads() -> int:
    return int(lib().oracle_threads())


def rel(x: np.ndarray, ref: np.ndarray) -> float:
    """max|x - ref| / max|ref| (tests/test_f16acc.py:11-12); NaN propagates."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ref = np.ascontiguousarray(ref, dtype=np.float64)
    if x.shape != ref.shape:
        raise ValueError("shape mismatch")
    return float(lib().oracle_rel(x.ctypes.data, ref.ctypes.data, x.size))
