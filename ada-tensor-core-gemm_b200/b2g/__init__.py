"""Python binding of libb200gemm.so, the B200 (sm_100a) FP16 tensor-core GEMM.

A thin ctypes layer over the C-ABI declared in ``include/b2g.h``. Device memory, streams
and process groups come from PyTorch when it is used; the arithmetic is in the library's
own sm_100a kernels. There is no fallback: if the library or a CUDA device is missing,
calls raise ``B2GError``.

The reference (RutwikPandit/ada-tensor-core-gemm) exposes its GEMM through the
``gemm_bench`` CLI (src/gemm_bench.cu:698-868); :func:`gemm` mirrors the launch it wraps
(``gemm_kernel(A, B, D, bias, M, N, K, alpha, group)``, src/gemm_bench.cu:215-217) with
the compile-time switches of that file (accumulate type, fused epilogue) as arguments.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(PKG_ROOT, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libb200gemm.so")
CSRC = os.path.join(PKG_ROOT, "csrc")

# b2g_status
OK, ERR_ARG, ERR_ALIGN, ERR_UNSUPPORTED, ERR_SMEM, ERR_CUDA, ERR_TIMEOUT, ERR_NO_DEVICE, \
    ERR_LIBRARY = range(9)
STATUS_NAMES = {0: "OK", 1: "ERR_ARG", 2: "ERR_ALIGN", 3: "ERR_UNSUPPORTED", 4: "ERR_SMEM",
                5: "ERR_CUDA", 6: "ERR_TIMEOUT", 7: "ERR_NO_DEVICE", 8: "ERR_LIBRARY"}

B_NK, B_KN = 0, 1
ACC_F32, ACC_F16 = 0, 1
EPI_NONE, EPI_BIAS_RELU = 0, 1
TILE_AUTO, TILE_128x128, TILE_128x256, TILE_256x256_2SM, TILE_128x64, TILE_256x512_2SM, \
    TILE_SWAP_AB, TILE_256x128_2SM = -1, 0, 1, 2, 3, 4, 5, 6

# Every symbol include/b2g.h declares (the CPU tests check the library exports them all).
EXPORTS = (
    "b2g_gemm", "b2g_last_error", "b2g_sync_status", "b2g_config_info", "b2g_cublas_gemm",
    "b2g_max_rel_diff", "b2g_bias_relu", "b2g_probe_tcgen05", "b2g_probe_hbm",
    "b2g_fill_lcg_f16", "b2g_fill_uniform_f16", "b2g_tile_coord",
    "b2g_selftest_wait_timeout", "b2g_set_wait_timeout_us", "b2g_version",
    "b2g_kernel_clock", "b2g_last_launch", "b2g_gemm_splitk", "b2g_gemm_splitk_noalloc",
    "b2g_gemm_multi", "b2g_allgather_rows", "b2g_gemm_multi_allgather", "b2g_gemm_peers",
    "b2g_ipc_handle", "b2g_ipc_open", "b2g_ipc_close", "b2g_last_launch_cluster",
    "b2g_last_launch_variant",
)


# b2g_last_launch_variant values (B2G_VARIANT_*)
VARIANT_NAMES = {0: "general", 1: "peers", 2: "plain", 3: "csplit", 4: "narrow"}


class B2GError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None


def build() -> None:
    """Compile the library and the gemm_bench CLI in-tree (nvcc for sm_100a)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", CSRC], check=True)


def lib():
    """Load libb200gemm.so (built in-tree by ``build()``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise B2GError(ERR_LIBRARY, f"{LIB_PATH} not built; run b2g.build()")
        L = C.CDLL(LIB_PATH)
        vp, i, ll, f, d = C.c_void_p, C.c_int, C.c_longlong, C.c_float, C.c_double
        L.b2g_gemm.restype = i
        L.b2g_gemm.argtypes = [vp, vp, vp, vp, i, i, i, ll, ll, ll, i, i, i, f, i, i, i, vp]
        L.b2g_gemm_splitk.restype = i
        L.b2g_gemm_splitk.argtypes = [vp, vp, vp, vp, i, i, i, ll, ll, ll, i, i, i, f, i, i, i,
                                      i, vp]
        L.b2g_gemm_splitk_noalloc.restype = i
        L.b2g_gemm_splitk_noalloc.argtypes = L.b2g_gemm_splitk.argtypes
        L.b2g_last_error.restype = C.c_char_p
        L.b2g_last_error.argtypes = []
        L.b2g_sync_status.restype = i
        L.b2g_sync_status.argtypes = [vp]
        L.b2g_config_info.restype = i
        ip = C.POINTER(C.c_int)
        L.b2g_config_info.argtypes = [i, i, ip, ip, ip, ip, ip, ip]
        L.b2g_cublas_gemm.restype = i
        L.b2g_cublas_gemm.argtypes = [vp, vp, vp, i, i, i, vp]
        L.b2g_max_rel_diff.restype = i
        L.b2g_max_rel_diff.argtypes = [vp, vp, C.c_size_t, vp, vp]
        L.b2g_bias_relu.restype = i
        L.b2g_bias_relu.argtypes = [vp, vp, i, i, ll, f, vp]
        L.b2g_probe_tcgen05.restype = i
        L.b2g_probe_tcgen05.argtypes = [i, i, i, i, C.POINTER(d), C.POINTER(C.c_longlong)]
        L.b2g_probe_hbm.restype = i
        L.b2g_probe_hbm.argtypes = [vp, vp, C.c_size_t, i, vp, C.POINTER(d)]
        L.b2g_fill_lcg_f16.restype = None
        L.b2g_fill_lcg_f16.argtypes = [vp, ll, vp, ll, vp, ll]
        L.b2g_fill_uniform_f16.restype = None
        L.b2g_fill_uniform_f16.argtypes = [vp, ll, ll, C.c_uint64, C.c_uint32, d, d]
        L.b2g_tile_coord.restype = None
        L.b2g_tile_coord.argtypes = [i, i, i, i, ip, ip]
        L.b2g_selftest_wait_timeout.restype = i
        L.b2g_selftest_wait_timeout.argtypes = [C.c_uint, vp]
        L.b2g_set_wait_timeout_us.restype = C.c_ulonglong
        L.b2g_set_wait_timeout_us.argtypes = [C.c_ulonglong]
        L.b2g_version.restype = i
        L.b2g_version.argtypes = []
        L.b2g_kernel_clock.restype = i
        L.b2g_kernel_clock.argtypes = [C.POINTER(d), C.POINTER(d)]
        L.b2g_last_launch.restype = i
        L.b2g_last_launch.argtypes = [ip, ip, ip, ip, ip, ip]
        L.b2g_last_launch_cluster.restype = i
        L.b2g_last_launch_cluster.argtypes = [ip]
        L.b2g_last_launch_variant.restype = i
        L.b2g_last_launch_variant.argtypes = [ip]
        L.b2g_gemm_multi.restype = i
        L.b2g_gemm_multi.argtypes = [i, ip, vp, vp, vp, vp, i, i, i, ll, ll, ll, i, i, i, f, i,
                                     i, i, vp, i]
        L.b2g_allgather_rows.restype = i
        L.b2g_allgather_rows.argtypes = [i, ip, vp, vp, i, i, ll, vp, i]
        L.b2g_gemm_multi_allgather.restype = i
        L.b2g_gemm_multi_allgather.argtypes = L.b2g_gemm_multi.argtypes
        L.b2g_gemm_peers.restype = i
        L.b2g_gemm_peers.argtypes = [vp, vp, vp, vp, i, i, i, ll, ll, ll, i, i, i, f, i, i, i,
                                     vp, i, vp]
        L.b2g_ipc_handle.restype = i
        L.b2g_ipc_handle.argtypes = [vp, vp, C.POINTER(C.c_ulonglong)]
        L.b2g_ipc_open.restype = i
        L.b2g_ipc_open.argtypes = [vp, C.POINTER(vp)]
        L.b2g_ipc_close.restype = i
        L.b2g_ipc_close.argtypes = [vp]
        _lib = L
    return _lib


def last_error() -> str:
    return lib().b2g_last_error().decode()


def _check(code: int) -> None:
    if code != OK:
        raise B2GError(code, last_error())


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream_ptr(stream) -> int | None:
    if stream is None:
        try:
            import torch

            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ---------------------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------------------
def gemm_raw(A: int, B: int, D: int, bias: int | None, M: int, N: int, K: int, lda: int,
             ldb: int, ldd: int, b_layout: int = B_NK, acc: int = ACC_F32,
             epilogue: int = EPI_NONE, alpha: float = 1.0, tile: int = TILE_AUTO,
             stages: int = 0, group: int = 1, stream: int | None = None,
             splits: int | None = None) -> None:
    """Launch D = A * B on raw device pointers (asynchronous). Raises B2GError.

    splits None: b2g_gemm (automatic split-K); an int: b2g_gemm_splitk with that factor
    (0 automatic, 1 none, S >= 2 forced)."""
    if splits is None:
        _check(lib().b2g_gemm(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue,
                              alpha, tile, stages, group, stream))
    else:
        _check(lib().b2g_gemm_splitk(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc,
                                     epilogue, alpha, tile, stages, group, splits, stream))


def gemm(A, B, D, bias=None, *, b_layout: int = B_NK, acc: int = ACC_F32,
         epilogue: int = EPI_NONE, alpha: float = 1.0, tile: int = TILE_AUTO,
         stages: int = 0, group: int = 1, stream=None, splits: int | None = None) -> None:
    """D = A * B (+ optional alpha*acc + bias + ReLU) on CUDA FP16 tensors.

    A: M x K, B: N x K (b_layout B_NK, the reference's TN layout) or K x N (B_KN),
    D: M x N; all row-major with unit inner stride (row pitch = stride(0)).
    """
    M, K = A.shape
    N = B.shape[0] if b_layout == B_NK else B.shape[1]
    for t, name in ((A, "A"), (B, "B"), (D, "D")):
        if t.stride(1) != 1:
            raise B2GError(ERR_ARG, f"{name} must have unit inner stride")
    if tuple(D.shape) != (M, N):
        raise B2GError(ERR_ARG, f"D shape {tuple(D.shape)} != ({M}, {N})")
    gemm_raw(_ptr(A), _ptr(B), _ptr(D), _ptr(bias), M, N, K, A.stride(0), B.stride(0),
             D.stride(0), b_layout, acc, epilogue, alpha, tile, stages, group,
             _stream_ptr(stream), splits)


def gemm_noalloc(A, B, D, bias=None, *, b_layout: int = B_NK, acc: int = ACC_F32,
                 epilogue: int = EPI_NONE, alpha: float = 1.0, tile: int = TILE_AUTO,
                 stages: int = 0, group: int = 1, stream=None, splits: int = 0) -> None:
    """:func:`gemm` through b2g_gemm_splitk_noalloc: no device memory is allocated; split-K
    uses the library's fixed static scratch (B2GError ERR_ARG if a split needs more).
    Calls that can overlap on one device share that scratch, so serialise them."""
    M, K = A.shape
    N = B.shape[0] if b_layout == B_NK else B.shape[1]
    if tuple(D.shape) != (M, N):
        raise B2GError(ERR_ARG, f"D shape {tuple(D.shape)} != ({M}, {N})")
    _check(lib().b2g_gemm_splitk_noalloc(_ptr(A), _ptr(B), _ptr(D), _ptr(bias), M, N, K,
                                         A.stride(0), B.stride(0), D.stride(0), b_layout, acc,
                                         epilogue, alpha, tile, stages, group, splits,
                                         _stream_ptr(stream)))


def _ptr_array(xs):
    return (C.c_void_p * len(xs))(*[_ptr(x) for x in xs])


def _devices_array(devices):
    return (C.c_int * len(devices))(*devices)


# rows [r0, r1) that device g of ngpu computes in gemm_multi (the C library's split)
from .shard import panel as panel_rows  # noqa: E402


def gemm_multi(A, B, D, bias=None, *, M: int, devices, b_layout: int = B_NK,
               acc: int = ACC_F32, epilogue: int = EPI_NONE, alpha: float = 1.0,
               tile: int = TILE_AUTO, stages: int = 0, group: int = 1, streams=None,
               sync: bool = True) -> None:
    """b2g_gemm_multi: one M x N x K GEMM split by M-row panels over ``devices``.

    A, D: per-device panels (rows from :func:`panel_rows`), B: per-device full copies, bias:
    per-device copies or None, streams: per-device streams or None. Row pitches are taken from
    the first device's tensors and must agree on every device."""
    ngpu = len(devices)
    if not (len(A) == len(B) == len(D) == ngpu) or (bias is not None and len(bias) != ngpu):
        raise B2GError(ERR_ARG, "one A panel, B copy, D panel (and bias) per device")
    K = A[0].shape[1]
    N = B[0].shape[0] if b_layout == B_NK else B[0].shape[1]
    for g in range(ngpu):
        r0, r1 = panel_rows(M, ngpu, g)
        if A[g].shape[0] != r1 - r0 or tuple(D[g].shape) != (r1 - r0, N):
            raise B2GError(ERR_ARG, f"device {g}: panel rows must be {r1 - r0}")
        if (A[g].stride(0), B[g].stride(0), D[g].stride(0)) != \
                (A[0].stride(0), B[0].stride(0), D[0].stride(0)):
            raise B2GError(ERR_ARG, f"device {g}: row pitches differ from device 0")
    sp = None if streams is None else _ptr_array([_stream_ptr(s) for s in streams])
    _check(lib().b2g_gemm_multi(ngpu, _devices_array(devices), _ptr_array(A), _ptr_array(B),
                                _ptr_array(D), None if bias is None else _ptr_array(bias), M, N,
                                K, A[0].stride(0), B[0].stride(0), D[0].stride(0), b_layout, acc,
                                epilogue, alpha, tile, stages, group, sp, int(sync)))


def allgather_rows(D, D_full, *, devices, streams=None, sync: bool = True) -> None:
    """b2g_allgather_rows: copy every device's D panel into every device's M x N ``D_full``
    over peer-to-peer copies."""
    ngpu = len(devices)
    if not (len(D) == len(D_full) == ngpu):
        raise B2GError(ERR_ARG, "one D panel and one D_full per device")
    M, N = D_full[0].shape
    ldd = D_full[0].stride(0)
    for g in range(ngpu):
        if D[g].stride(0) != ldd or D_full[g].stride(0) != ldd:
            raise B2GError(ERR_ARG, "D panels and D_full must share one row pitch")
    sp = None if streams is None else _ptr_array([_stream_ptr(s) for s in streams])
    _check(lib().b2g_allgather_rows(ngpu, _devices_array(devices), _ptr_array(D),
                                    _ptr_array(D_full), M, N, ldd, sp, int(sync)))


def gemm_multi_allgather(A, B, D_full, bias=None, *, devices, b_layout: int = B_NK,
                         acc: int = ACC_F32, epilogue: int = EPI_NONE, alpha: float = 1.0,
                         tile: int = TILE_AUTO, stages: int = 0, group: int = 1, streams=None,
                         sync: bool = True) -> None:
    """b2g_gemm_multi_allgather: the M-panel GEMM with the all-gather fused into its epilogue.

    A: per-device panels (rows from :func:`panel_rows`), B: per-device full copies, D_full:
    one M x N matrix per device, each receiving every device's rows."""
    ngpu = len(devices)
    if not (len(A) == len(B) == len(D_full) == ngpu) or (bias is not None and len(bias) != ngpu):
        raise B2GError(ERR_ARG, "one A panel, B copy, D_full (and bias) per device")
    M, N = D_full[0].shape
    K = A[0].shape[1]
    for g in range(ngpu):
        r0, r1 = panel_rows(M, ngpu, g)
        if A[g].shape[0] != r1 - r0 or tuple(D_full[g].shape) != (M, N):
            raise B2GError(ERR_ARG, f"device {g}: A panel rows {r1 - r0}, D_full {M} x {N}")
        if (A[g].stride(0), B[g].stride(0), D_full[g].stride(0)) != \
                (A[0].stride(0), B[0].stride(0), D_full[0].stride(0)):
            raise B2GError(ERR_ARG, f"device {g}: row pitches differ from device 0")
    sp = None if streams is None else _ptr_array([_stream_ptr(s) for s in streams])
    _check(lib().b2g_gemm_multi_allgather(
        ngpu, _devices_array(devices), _ptr_array(A), _ptr_array(B), _ptr_array(D_full),
        None if bias is None else _ptr_array(bias), M, N, K, A[0].stride(0), B[0].stride(0),
        D_full[0].stride(0), b_layout, acc, epilogue, alpha, tile, stages, group, sp, int(sync)))


def gemm_peers(A, B, D, peers, bias=None, *, b_layout: int = B_NK, acc: int = ACC_F32,
               epilogue: int = EPI_NONE, alpha: float = 1.0, tile: int = TILE_AUTO,
               stages: int = 0, group: int = 1, stream=None) -> None:
    """b2g_gemm_peers: D = A * B on this device, every element of D also stored into each of
    ``peers`` (raw device addresses of D's first row in other copies with D's row pitch,
    e.g. from :func:`ipc_open`)."""
    M, K = A.shape
    N = B.shape[0] if b_layout == B_NK else B.shape[1]
    if tuple(D.shape) != (M, N):
        raise B2GError(ERR_ARG, f"D shape {tuple(D.shape)} != ({M}, {N})")
    arr = (C.c_void_p * max(1, len(peers)))(*peers)
    _check(lib().b2g_gemm_peers(_ptr(A), _ptr(B), _ptr(D), _ptr(bias), M, N, K, A.stride(0),
                                B.stride(0), D.stride(0), b_layout, acc, epilogue, alpha, tile,
                                stages, group, arr, len(peers), _stream_ptr(stream)))


def ipc_handle(t) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding tensor/pointer t, t's byte offset)."""
    h = C.create_string_buffer(64)
    off = C.c_ulonglong()
    _check(lib().b2g_ipc_handle(_ptr(t), h, C.byref(off)))
    return h.raw, off.value


def ipc_open(handle: bytes) -> int:
    """Map another process's allocation; returns its base address in this process."""
    base = C.c_void_p()
    _check(lib().b2g_ipc_open(C.create_string_buffer(handle, 64), C.byref(base)))
    return base.value


def ipc_close(base: int) -> None:
    _check(lib().b2g_ipc_close(base))


def sync_status(stream=None) -> None:
    """Synchronise the stream and raise B2GError if a device-side wait gave up."""
    _check(lib().b2g_sync_status(_stream_ptr(stream)))


def config_info(tile: int = TILE_AUTO, stages: int = 0) -> dict:
    vals = [C.c_int() for _ in range(6)]
    _check(lib().b2g_config_info(tile, stages, *[C.byref(v) for v in vals]))
    keys = ("threads", "regs", "smem", "ctas_per_sm", "tmem_cols", "stages")
    return {k: v.value for k, v in zip(keys, vals)}


def last_launch() -> dict:
    """Grid, threads, tile, stages, work units, split-K factor, cluster size and kernel
    variant ("plain", "csplit", "peers", "narrow" or "general") of this thread's most recent GEMM
    launch."""
    vals = [C.c_int() for _ in range(6)]
    _check(lib().b2g_last_launch(*[C.byref(v) for v in vals]))
    keys = ("grid", "threads", "tile", "stages", "units", "splits")
    out = {k: v.value for k, v in zip(keys, vals)}
    cl = C.c_int()
    _check(lib().b2g_last_launch_cluster(C.byref(cl)))
    out["cluster"] = cl.value  # CTAs per thread-block cluster (split-K clusters: the splits)
    var = C.c_int()
    _check(lib().b2g_last_launch_variant(C.byref(var)))
    out["variant"] = VARIANT_NAMES.get(var.value, var.value)  # compiled form of the kernel
    return out


def cublas_gemm(A, B, D, stream=None) -> None:
    """The reference's cuBLAS comparison call (B stored N x K)."""
    M, K = A.shape
    N = B.shape[0]
    _check(lib().b2g_cublas_gemm(_ptr(A), _ptr(B), _ptr(D), M, N, K, _stream_ptr(stream)))


def max_rel_diff(x, y, out_dev, stream=None) -> None:
    _check(lib().b2g_max_rel_diff(_ptr(x), _ptr(y), x.numel(), _ptr(out_dev),
                                  _stream_ptr(stream)))


def bias_relu(D, bias, alpha: float = 1.0, stream=None) -> None:
    M, N = D.shape
    _check(lib().b2g_bias_relu(_ptr(D), _ptr(bias), M, N, D.stride(0), alpha,
                               _stream_ptr(stream)))


PROBE_KINDS = {0: "f16 in / f32 acc", 1: "f16 in / f16 acc", 2: "s8 in / s32 acc",
               3: "e4m3 in / f32 acc"}


def probe_tcgen05(kind: int = 0, cta_group: int = 1, n: int = 256, iters: int = 4096):
    """(dense FLOP per clock per SM, cycles of the least-perturbed SM)."""
    fl, cy = C.c_double(), C.c_longlong()
    _check(lib().b2g_probe_tcgen05(kind, cta_group, n, iters, C.byref(fl), C.byref(cy)))
    return fl.value, cy.value


def probe_hbm(src, dst, nbytes: int, reps: int = 20, stream=None) -> float:
    g = C.c_double()
    _check(lib().b2g_probe_hbm(_ptr(src), _ptr(dst), nbytes, reps, _stream_ptr(stream),
                               C.byref(g)))
    return g.value


def fill_uniform(n: int, seed: int, tensor_id: int, lo: float = -1.0, hi: float = 1.0,
                 out=None, first: int = 0):
    """Seeded synthetic FP16 values for global indices first..first+n-1 (numpy uint16
    array, or written into `out`: a numpy array, a tensor or a host pointer)."""
    import numpy as np

    if out is None:
        out = np.empty(n, np.uint16)
    ptr = out.ctypes.data if hasattr(out, "ctypes") else _ptr(out)
    lib().b2g_fill_uniform_f16(ptr, n, first, seed, tensor_id, lo, hi)
    return out


def fill_lcg(M: int, N: int, K: int):
    """The reference's deterministic init: (A M x K, B N x K, bias N) as numpy uint16."""
    import numpy as np

    A = np.empty((M, K), np.uint16)
    B = np.empty((N, K), np.uint16)
    bias = np.empty(N, np.uint16)
    lib().b2g_fill_lcg_f16(A.ctypes.data, A.size, B.ctypes.data, B.size, bias.ctypes.data,
                           bias.size)
    return A, B, bias


def tile_coord(linear: int, tiles_m: int, tiles_n: int, group: int):
    m, n = C.c_int(), C.c_int()
    lib().b2g_tile_coord(linear, tiles_m, tiles_n, group, C.byref(m), C.byref(n))
    return m.value, n.value


def selftest_wait_timeout(timeout_us: int = 20000, stream=None) -> int:
    """Run the bounded-wait self-test; returns the status code (ERR_TIMEOUT when working)."""
    return lib().b2g_selftest_wait_timeout(timeout_us, _stream_ptr(stream))


def set_wait_timeout_us(us: int) -> int:
    return int(lib().b2g_set_wait_timeout_us(us))


def version() -> int:
    return int(lib().b2g_version())


def kernel_clock():
    """(SM MHz, CTA-0 lifetime in us) of the most recent completed GEMM launch."""
    mhz, us = C.c_double(), C.c_double()
    _check(lib().b2g_kernel_clock(C.byref(mhz), C.byref(us)))
    return mhz.value, us.value
