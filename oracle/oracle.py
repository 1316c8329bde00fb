"""CPU oracle for the FP16 GEMM hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference leg of
``bench.py`` may import this module, and only as the checker (or the timed CPU baseline).
The product path never imports it.

This is a thin numpy/ctypes layer over ``oracle/liboracle.so`` (``oracle/oracle.c``), which
restates the reference's algorithm (citations are in the C file), and over
``oracle/_ref/libref.so`` -- the reference's own code compiled from its unmodified source
(``oracle/ref_shim.cu``) -- when that library is present.

FP16 arrays are numpy ``uint16`` bit patterns (or ``float16`` views of them).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libref.so")

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_ip = C.POINTER(C.c_int)

_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference checkout exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_f16_array.argtypes = [_f32p, _u16p, C.c_int64]
        L.orc_f16_to_f32_array.argtypes = [_u16p, _f32p, C.c_int64]
        L.orc_fill_lcg.argtypes = [_u16p, C.c_int64, _u16p, C.c_int64, _u16p, C.c_int64]
        L.orc_fill_uniform.argtypes = [_u16p, C.c_int64, C.c_int64, C.c_uint64, C.c_uint32,
                                       C.c_double, C.c_double]
        L.orc_gemm_f64.argtypes = [_u16p, C.c_int64, _u16p, C.c_int64, C.c_int, C.c_int,
                                   C.c_int, C.c_int, C.c_int, C.c_int, _f64p]
        L.orc_gemm_f32_naive.argtypes = [_u16p, C.c_int64, _u16p, C.c_int64, C.c_int, C.c_int,
                                         C.c_int, C.c_int, _f32p]
        L.orc_gemm_f32_blocked.restype = C.c_int
        L.orc_gemm_f32_blocked.argtypes = [_u16p, C.c_int64, _u16p, C.c_int64, C.c_int,
                                           C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_spot_check.restype = C.c_double
        L.orc_spot_check.argtypes = [_u16p, _u16p, _u16p, C.c_void_p, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_int, C.c_float, _ip, _ip]
        L.orc_max_rel_diff.restype = C.c_float
        L.orc_max_rel_diff.argtypes = [_u16p, _u16p, C.c_int64]
        L.orc_frobenius_rel.restype = C.c_double
        L.orc_frobenius_rel.argtypes = [_u16p, C.c_int64, _f64p, C.c_int, C.c_int]
        L.orc_tile_coord.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _ip, _ip]
        L.orc_epilogue.restype = C.c_uint16
        L.orc_epilogue.argtypes = [C.c_float, C.c_int, C.c_float, C.c_uint16, C.c_int]
        L.orc_epilogue_array.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_float,
                                         C.c_void_p, _u16p]
        L.orc_bias_relu.argtypes = [_u16p, C.c_void_p, C.c_int, C.c_int, C.c_float]
        L.orc_num_threads.restype = C.c_int
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own code (oracle/_ref/libref.so), or None if it was not built."""
    global _ref
    if _ref is None and ref_available():
        R = C.CDLL(REF_PATH)
        R.ref_spot_check.restype = C.c_double
        R.ref_spot_check.argtypes = [_u16p, _u16p, _u16p, C.c_void_p, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_int, C.c_float, _ip, _ip]
        R.ref_float2half.restype = C.c_uint16
        R.ref_float2half.argtypes = [C.c_float]
        R.ref_gemm_launch.restype = C.c_int
        R.ref_gemm_launch.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_void_p]
        R.ref_max_rel_diff.restype = C.c_int
        R.ref_max_rel_diff.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                       C.c_void_p]
        R.ref_bias_relu.restype = C.c_int
        R.ref_bias_relu.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float,
                                    C.c_void_p]
        R.ref_cpu_rows.restype = C.c_double
        R.ref_cpu_rows.argtypes = [_u16p, _u16p, _u16p, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_int]
        _ref = R
    return _ref


# ---------------------------------------------------------------------------------------
# numpy helpers
# ---------------------------------------------------------------------------------------
def _u16(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def f32_to_f16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16_array(x.reshape(-1), out.reshape(-1), x.size)
    return out


def f16_to_f32(h) -> np.ndarray:
    h = _u16(h)
    out = np.empty(h.shape, np.float32)
    lib().orc_f16_to_f32_array(h.reshape(-1), out.reshape(-1), h.size)
    return out


def fill_lcg(M: int, N: int, K: int):
    """A (M x K), B (N x K), bias (N) exactly as the reference initialises them."""
    A = np.empty((M, K), np.uint16)
    B = np.empty((N, K), np.uint16)
    bias = np.empty((N,), np.uint16)
    lib().orc_fill_lcg(A.reshape(-1), A.size, B.reshape(-1), B.size, bias, bias.size)
    return A, B, bias


def fill_uniform(shape, seed: int, tensor_id: int, lo: float = -1.0, hi: float = 1.0,
                 first: int = 0):
    out = np.empty(shape, np.uint16)
    lib().orc_fill_uniform(out.reshape(-1), out.size, first, seed, tensor_id, lo, hi)
    return out


def gemm_f64(A, B, b_layout: int = 0, m0: int = 0, m1: int | None = None) -> np.ndarray:
    """FP64 reference of rows [m0, m1). A: M x K. B: N x K (layout 0) or K x N (layout 1)."""
    A, B = _u16(A), _u16(B)
    M, K = A.shape
    N = B.shape[0] if b_layout == 0 else B.shape[1]
    m1 = M if m1 is None else m1
    out = np.empty((m1 - m0, N), np.float64)
    lib().orc_gemm_f64(A.reshape(-1), A.shape[1], B.reshape(-1), B.shape[1], b_layout, M, N,
                       K, m0, m1, out.reshape(-1))
    return out


def gemm_f32_naive(A, B, b_layout: int = 0) -> np.ndarray:
    A, B = _u16(A), _u16(B)
    M, K = A.shape
    N = B.shape[0] if b_layout == 0 else B.shape[1]
    out = np.empty((M, N), np.float32)
    lib().orc_gemm_f32_naive(A.reshape(-1), A.shape[1], B.reshape(-1), B.shape[1], b_layout,
                             M, N, K, out.reshape(-1))
    return out


def gemm_f32_blocked(A, B, b_layout: int = 0, m0: int = 0, m1: int | None = None):
    """Blocked FP32 CPU GEMM (the bench's CPU baseline). Returns (D32 rows, threads)."""
    A, B = _u16(A), _u16(B)
    M, K = A.shape
    N = B.shape[0] if b_layout == 0 else B.shape[1]
    m1 = M if m1 is None else m1
    out = np.empty((m1 - m0, N), np.float32)
    t = lib().orc_gemm_f32_blocked(A.reshape(-1), A.shape[1], B.reshape(-1), B.shape[1],
                                   b_layout, M, N, K, m0, m1, out.reshape(-1))
    return out, t


def spot_check(A, B, D, bias=None, samples: int = 512, fused: bool = False,
               alpha: float = 1.0):
    """Restated cpu_spot_check: (worst_rel, worst_m, worst_n). B is N x K."""
    A, B, D = _u16(A), _u16(B), _u16(D)
    M, K = A.shape
    N = B.shape[0]
    wm, wn = C.c_int(), C.c_int()
    b = None if bias is None else _u16(bias)
    w = lib().orc_spot_check(A.reshape(-1), B.reshape(-1), D.reshape(-1),
                             None if b is None else b.ctypes.data, M, N, K, samples,
                             int(fused), alpha, C.byref(wm), C.byref(wn))
    return w, wm.value, wn.value


def ref_spot_check(A, B, D, bias=None, samples: int = 512, fused: bool = False,
                   alpha: float = 1.0):
    """The reference's own cpu_spot_check (compiled from its source)."""
    A, B, D = _u16(A), _u16(B), _u16(D)
    M, K = A.shape
    N = B.shape[0]
    wm, wn = C.c_int(), C.c_int()
    b = None if bias is None else _u16(bias)
    w = ref().ref_spot_check(A.reshape(-1), B.reshape(-1), D.reshape(-1),
                             None if b is None else b.ctypes.data, M, N, K, samples,
                             int(fused), alpha, C.byref(wm), C.byref(wn))
    return w, wm.value, wn.value


def max_rel_diff(x, y) -> float:
    x, y = _u16(x), _u16(y)
    return float(lib().orc_max_rel_diff(x.reshape(-1), y.reshape(-1), x.size))


def frobenius_rel(D, R) -> float:
    D = _u16(D)
    R = np.ascontiguousarray(R, dtype=np.float64)
    M, N = R.shape
    return float(lib().orc_frobenius_rel(D.reshape(-1), D.shape[1], R.reshape(-1), M, N))


def tile_coord(linear: int, tiles_m: int, tiles_n: int, group: int):
    m, n = C.c_int(), C.c_int()
    lib().orc_tile_coord(linear, tiles_m, tiles_n, group, C.byref(m), C.byref(n))
    return m.value, n.value


def epilogue(acc32, bias=None, alpha: float = 1.0, fused: bool = True) -> np.ndarray:
    """Apply the reference epilogue to an FP32 accumulator matrix -> FP16 bits."""
    acc32 = np.ascontiguousarray(acc32, dtype=np.float32)
    M, N = acc32.shape
    out = np.empty((M, N), np.uint16)
    b = None if bias is None else _u16(bias)
    lib().orc_epilogue_array(acc32.reshape(-1), M, N, int(fused), alpha,
                             None if b is None else b.ctypes.data, out.reshape(-1))
    return out


def bias_relu(D, bias, alpha: float = 1.0) -> np.ndarray:
    D = _u16(D).copy()
    M, N = D.shape
    b = None if bias is None else _u16(bias)
    lib().orc_bias_relu(D.reshape(-1), None if b is None else b.ctypes.data, M, N, alpha)
    return D


def num_threads() -> int:
    return int(lib().orc_num_threads())
