"""CPU tests of the C-ABI library: it loads without a GPU, exports every symbol that
include/b2g.h declares, validates arguments before touching the device, and its host
logic (tile scheduler, input generators) agrees with the oracle."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import b2g
import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b2g.h")
CLI = os.path.join(b2g.LIB_DIR, "gemm_bench")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2g_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = b2g.lib()
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(L, s), f"{s} declared in b2g.h but not exported"
    assert set(syms) == set(b2g.EXPORTS)


def test_version_and_last_error():
    assert b2g.version() >= 100
    assert isinstance(b2g.last_error(), str)


def test_argument_validation_without_gpu():
    L = b2g.lib()
    # bad arguments are rejected before any CUDA call
    assert L.b2g_gemm(None, None, None, None, -1, 4, 4, 4, 4, 4, 0, 0, 0, 1.0, -1, 0, 1,
                      None) == b2g.ERR_ARG
    assert "negative" in b2g.last_error()
    assert L.b2g_gemm(None, None, None, None, 4, 4, 4, 8, 8, 4, 5, 0, 0, 1.0, -1, 0, 1,
                      None) == b2g.ERR_ARG
    assert L.b2g_gemm(None, None, None, None, 4, 4, 4, 8, 8, 4, 0, 2, 0, 1.0, -1, 0, 1,
                      None) == b2g.ERR_ARG
    assert L.b2g_gemm(None, None, None, None, 4, 4, 4, 8, 8, 4, 0, 0, 0, 1.0, 7, 0, 1,
                      None) == b2g.ERR_ARG
    assert L.b2g_gemm(None, None, None, None, 4, 4, 4, 8, 8, 4, 0, 0, 0, 1.0, -1, 9, 1,
                      None) == b2g.ERR_ARG
    # empty problems are a no-op
    assert L.b2g_gemm(None, None, None, None, 0, 4, 4, 8, 8, 4, 0, 0, 0, 1.0, -1, 0, 1,
                      None) == b2g.OK
    # a valid call on a machine without a device fails cleanly
    rc = L.b2g_gemm(16, 16, 16, None, 4, 4, 8, 8, 8, 4, 0, 0, 0, 1.0, -1, 0, 1, None)
    assert rc in (b2g.ERR_NO_DEVICE, b2g.OK)
    assert L.b2g_selftest_wait_timeout(0, None) == b2g.ERR_ARG
    assert L.b2g_probe_tcgen05(7, 1, 256, 10, None, None) == b2g.ERR_ARG


def test_tile_coord_matches_reference_rasterization():
    for tm, tn, g in [(1, 1, 1), (7, 5, 1), (7, 5, 2), (7, 5, 3), (32, 16, 8), (33, 17, 16),
                      (3, 100, 16), (256, 256, 8)]:
        seen = set()
        for t in range(tm * tn):
            got = b2g.tile_coord(t, tm, tn, g)
            assert got == O.tile_coord(t, tm, tn, g)
            seen.add(got)
        assert len(seen) == tm * tn


def test_generators_match_oracle():
    for seed, tid, lo, hi in [(0, 0, -1.0, 1.0), (1, 1, -1.0, 1.0), (2, 0, -0.5, 0.5),
                              (12345, 2, -0.3, 0.7)]:
        got = b2g.fill_uniform(100003, seed, tid, lo, hi)
        assert np.array_equal(got, O.fill_uniform((100003,), seed, tid, lo, hi))
    A, B, bias = b2g.fill_lcg(33, 17, 40)
    A2, B2, bias2 = O.fill_lcg(33, 17, 40)
    assert np.array_equal(A, A2) and np.array_equal(B, B2) and np.array_equal(bias, bias2)


def test_wait_timeout_setting():
    prev = b2g.set_wait_timeout_us(1234567)
    assert b2g.set_wait_timeout_us(prev) == 1234567


def test_cli_flags_without_gpu():
    assert os.path.exists(CLI)
    r = subprocess.run([CLI, "--help"], capture_output=True, text=True)
    assert r.returncode == 0 and "--tile" in r.stdout and "--soak" in r.stdout
    r = subprocess.run([CLI, "--definitely-not-a-flag"], capture_output=True, text=True)
    assert r.returncode == 2 and "unknown option" in r.stderr
    r = subprocess.run([CLI, "--acc", "f64"], capture_output=True, text=True)
    assert r.returncode == 2


def test_generator_panels_are_slices_of_the_full_matrix():
    full = b2g.fill_uniform(64 * 48, 3, 0)
    for first, n in [(0, 100), (48 * 10, 48 * 7), (64 * 48 - 5, 5)]:
        assert np.array_equal(b2g.fill_uniform(n, 3, 0, first=first), full[first:first + n])
        assert np.array_equal(O.fill_uniform((n,), 3, 0, first=first), full[first:first + n])


def test_splitk_argument_validation_without_gpu():
    """b2g_gemm_splitk / _noalloc reject bad split requests before touching the device."""
    L = b2g.lib()
    for fn in (L.b2g_gemm_splitk, L.b2g_gemm_splitk_noalloc):  # argtypes set by b2g.lib()
        args = [None, None, None, None, 4, 4, 64, 64, 64, 4, 0, 0, 0, 1.0, -1, 0, 1]
        assert fn(*args, -1, None) == b2g.ERR_ARG           # negative split factor
        assert "splits" in b2g.last_error()
        acc16 = list(args)
        acc16[11] = b2g.ACC_F16
        assert fn(*acc16, 2, None) == b2g.ERR_UNSUPPORTED    # split-K needs FP32 accumulation
        bad_tile = list(args)
        bad_tile[14] = 7
        assert fn(*bad_tile, 0, None) == b2g.ERR_ARG         # tiles are -1 .. 6


def test_last_launch_before_any_launch():
    """b2g_last_launch reports an error on a thread that has launched nothing."""
    import threading

    out = {}

    def probe():
        try:
            b2g.last_launch()
            out["rc"] = b2g.OK
        except b2g.B2GError as e:
            out["rc"] = e.code

    t = threading.Thread(target=probe)
    t.start()
    t.join()
    assert out["rc"] == b2g.ERR_ARG


def test_multi_gpu_argument_validation_without_gpu():
    """b2g_gemm_multi / b2g_allgather_rows reject bad arguments before touching any device."""
    L = b2g.lib()
    dev = (C.c_int * 1)(0)
    ptrs = (C.c_void_p * 1)(None)
    tail = [64, 64, 64, 64, 64, 64, 0, 0, 0, 1.0, -1, 0, 1, None, 1]
    assert L.b2g_gemm_multi(0, dev, ptrs, ptrs, ptrs, None, *tail) == b2g.ERR_ARG
    assert "ngpu" in b2g.last_error()
    assert L.b2g_gemm_multi(1, None, ptrs, ptrs, ptrs, None, *tail) == b2g.ERR_ARG
    neg = [-1] + tail[1:]
    assert L.b2g_gemm_multi(1, dev, ptrs, ptrs, ptrs, None, *neg) == b2g.ERR_ARG
    fused = L.b2g_gemm_multi_allgather
    assert fused(0, dev, ptrs, ptrs, ptrs, None, *tail) == b2g.ERR_ARG
    devs9 = (C.c_int * 9)(*range(9))
    ptrs9 = (C.c_void_p * 9)()
    assert fused(9, devs9, ptrs9, ptrs9, ptrs9, None, *tail) == b2g.ERR_ARG  # 8 devices at most
    assert fused(1, dev, ptrs, ptrs, ptrs, None, *neg) == b2g.ERR_ARG
    assert fused(1, dev, ptrs, ptrs, ptrs, None, *tail) == b2g.ERR_ARG      # D_full[0] NULL
    assert "D_full" in b2g.last_error()
    assert L.b2g_allgather_rows(0, dev, ptrs, ptrs, 64, 64, 64, None, 1) == b2g.ERR_ARG
    assert L.b2g_allgather_rows(1, dev, ptrs, None, 64, 64, 64, None, 1) == b2g.ERR_ARG
    assert L.b2g_allgather_rows(1, dev, ptrs, ptrs, 64, 64, 32, None, 1) == b2g.ERR_ARG
    assert "ldd" in b2g.last_error()



def test_multi_gpu_without_a_device():
    """With well-formed arguments the multi-device entry points ask the runtime for devices
    first; here (no GPU) that is B2G_ERR_NO_DEVICE, returned without starting any work."""
    L = b2g.lib()
    dev = (C.c_int * 1)(0)
    fake = (C.c_void_p * 1)(0x1000)
    tail = [64, 64, 64, 64, 64, 64, 0, 0, 0, 1.0, -1, 0, 1, None, 1]
    assert L.b2g_gemm_multi(1, dev, fake, fake, fake, None, *tail) == b2g.ERR_NO_DEVICE
    assert L.b2g_gemm_multi_allgather(1, dev, fake, fake, fake, None, *tail) == b2g.ERR_NO_DEVICE
    assert L.b2g_allgather_rows(1, dev, fake, fake, 64, 64, 64, None, 1) == b2g.ERR_NO_DEVICE
    assert "no CUDA device" in b2g.last_error()


def test_peers_and_ipc_argument_validation_without_gpu():
    L = b2g.lib()
    args = [None, None, None, None, 64, 64, 64, 64, 64, 64, 0, 0, 0, 1.0, -1, 0, 1]
    assert L.b2g_gemm_peers(*args, None, -1, None) == b2g.ERR_ARG
    assert L.b2g_gemm_peers(*args, None, 8, None) == b2g.ERR_ARG       # 7 copies at most
    assert L.b2g_gemm_peers(*args, None, 2, None) == b2g.ERR_ARG       # peer_D NULL
    off = C.c_ulonglong()
    buf = C.create_string_buffer(64)
    assert L.b2g_ipc_handle(None, buf, C.byref(off)) == b2g.ERR_ARG
    base = C.c_void_p()
    assert L.b2g_ipc_open(None, C.byref(base)) == b2g.ERR_ARG
    assert L.b2g_ipc_close(None) == b2g.ERR_ARG


def test_multi_gpu_python_wrappers_validate_on_the_host():
    """The Python wrappers check panel shapes and pitches before calling the library; with
    consistent CPU tensors the call reaches the library, which finds no device here."""
    import torch

    M, N, K = 10, 16, 8
    devs = [0, 0]
    A = [torch.zeros(5, K, dtype=torch.float16), torch.zeros(5, K, dtype=torch.float16)]
    B = [torch.zeros(N, K, dtype=torch.float16)] * 2
    D = [torch.zeros(5, N, dtype=torch.float16), torch.zeros(5, N, dtype=torch.float16)]
    full = [torch.zeros(M, N, dtype=torch.float16)] * 2
    with pytest.raises(b2g.B2GError, match="panel rows"):
        b2g.gemm_multi([A[0], torch.zeros(4, K, dtype=torch.float16)], B, D, M=M, devices=devs)
    with pytest.raises(b2g.B2GError, match="per device"):
        b2g.gemm_multi(A[:1], B, D, M=M, devices=devs)
    with pytest.raises(b2g.B2GError, match="pitches"):
        wide = torch.zeros(5, K + 8, dtype=torch.float16)[:, :K]
        b2g.gemm_multi([A[0], wide], B, D, M=M, devices=devs)
    with pytest.raises(b2g.B2GError) as e:
        b2g.gemm_multi(A, B, D, M=M, devices=devs)
    assert e.value.code == b2g.ERR_NO_DEVICE
    with pytest.raises(b2g.B2GError, match="A panel rows"):
        b2g.gemm_multi_allgather([A[0], A[0][:4]], B, full, devices=devs)
    with pytest.raises(b2g.B2GError) as e:
        b2g.gemm_multi_allgather(A, B, full, devices=devs)
    assert e.value.code == b2g.ERR_NO_DEVICE
    with pytest.raises(b2g.B2GError, match="one row pitch"):
        b2g.allgather_rows([torch.zeros(5, N + 8, dtype=torch.float16)[:, :N], D[1]], full,
                           devices=devs)
    with pytest.raises(b2g.B2GError, match="D shape"):
        b2g.gemm_peers(A[0], B[0], D[0][:4], [])
