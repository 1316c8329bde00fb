"""GPU tests of the one-process multi-device entry points b2g_gemm_multi (M-row panels, one
host thread per device), b2g_allgather_rows (peer-to-peer copies of the D panels) and
b2g_gemm_multi_allgather (the all-gather fused into the GEMM epilogue).

On a single-GPU box the "devices" list names device 0 more than once: every panel then runs
on device 0 from its own host thread and stream, which exercises the panel split, the threads
and the gather copies. Tests with two real devices run when two are visible."""
import subprocess

import numpy as np
import pytest

import b2g
from helpers import check_rows, inputs, run, sample_rows, to_dev, to_host

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _ndev():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _panels(A, B, bias, devices):
    """Per-device A panels, B copies, bias copies and empty D panels (NaN-filled)."""
    M = A.shape[0]
    N = B.shape[0]
    dA, dB, dBias, dD = [], [], [], []
    for g, dev in enumerate(devices):
        r0, r1 = b2g.panel_rows(M, len(devices), g)
        with torch.cuda.device(dev):
            dA.append(to_dev(torch, A[r0:r1]))
            dB.append(to_dev(torch, B))
            dBias.append(to_dev(torch, bias))
            dD.append(torch.full((r1 - r0, N), float("nan"), dtype=torch.float16,
                                 device=f"cuda:{dev}"))
    return dA, dB, dBias, dD


def _assemble(dD):
    return np.concatenate([to_host(d) for d in dD])


@pytest.mark.parametrize("devices", [[0], [0, 0], [0, 0, 0]])
@pytest.mark.parametrize("M,N,K", [(512, 384, 256), (1000, 520, 200), (3, 64, 64)])
def test_multi_matches_single_device(devices, M, N, K):
    """The panels of b2g_gemm_multi, stacked, equal one b2g_gemm of each panel, bit for bit,
    and the whole product agrees with the FP64 oracle."""
    A, B, bias = inputs(M, N, K, seed=M + N)
    dA, dB, _, dD = _panels(A, B, bias, devices)
    b2g.gemm_multi(dA, dB, dD, M=M, devices=devices)
    D = _assemble(dD)
    ref = np.concatenate([run(torch, A[r0:r1], B)
                          for r0, r1 in (b2g.panel_rows(M, len(devices), g)
                                         for g in range(len(devices))) if r1 > r0])
    assert np.array_equal(D, ref)
    frob, _ = check_rows(A, B, D, sample_rows(M, 64))
    assert frob <= 1e-3


def test_multi_fused_epilogue_and_streams():
    devices = [0, 0]
    M, N, K = 640, 256, 512
    A, B, bias = inputs(M, N, K, seed=7)
    dA, dB, dBias, dD = _panels(A, B, bias, devices)
    streams = [torch.cuda.Stream(device=d) for d in devices]
    b2g.gemm_multi(dA, dB, dD, dBias, M=M, devices=devices, epilogue=b2g.EPI_BIAS_RELU,
                   alpha=0.5, streams=streams, sync=False)
    for s in streams:
        s.synchronize()
    D = _assemble(dD)
    frob, maxrel = check_rows(A, B, D, sample_rows(M, 64), bias=bias, alpha=0.5, epilogue=True)
    assert frob <= 1e-3 and maxrel < 3e-2


def test_multi_names_the_failing_device():
    devices = [0, 0]
    M, N, K = 256, 128, 64
    A, B, bias = inputs(M, N, K)
    dA, dB, _, dD = _panels(A, B, bias, devices)
    L = b2g.lib()
    arr = lambda ts: (b2g.C.c_void_p * 2)(*[t.data_ptr() for t in ts])  # noqa: E731
    devs = (b2g.C.c_int * 2)(*devices)
    # lda < K is rejected by every device's launch; the message names the device and panel
    rc = L.b2g_gemm_multi(2, devs, arr(dA), arr(dB), arr(dD), None, M, N, K, K - 1, K, N, 0, 0,
                          0, 1.0, -1, 0, 1, None, 1)
    assert rc == b2g.ERR_ARG
    msg = b2g.last_error()
    assert "device 0" in msg and "lda" in msg


@pytest.mark.parametrize("devices", [[0], [0, 0], [0, 0, 0, 0]])
@pytest.mark.parametrize("N", [200, 203])
def test_allgather_rows(devices, N):
    """Every device's gathered copy equals the stacked panels, bit for bit (N % 8 == 0: the
    SM push kernel; else copy-engine 2D copies)."""
    M, K = 515, 128
    A, B, bias = inputs(M, N, K, seed=3)
    dA, dB, _, dD = _panels(A, B, bias, devices)
    b2g.gemm_multi(dA, dB, dD, M=M, devices=devices)
    full = [torch.full((M, N), float("nan"), dtype=torch.float16, device=f"cuda:{d}")
            for d in devices]
    b2g.allgather_rows(dD, full, devices=devices)
    D = _assemble(dD)
    for f in full:
        assert np.array_equal(to_host(f), D)


@pytest.mark.skipif(_ndev() < 2, reason="needs two devices")
def test_two_devices_gemm_and_allgather():
    devices = [0, 1]
    M, N, K = 2048, 1024, 512
    A, B, bias = inputs(M, N, K, seed=11)
    dA, dB, _, dD = _panels(A, B, bias, devices)
    b2g.gemm_multi(dA, dB, dD, M=M, devices=devices)
    D = _assemble(dD)
    assert np.array_equal(D[:M // 2], run(torch, A[:M // 2], B))
    frob, _ = check_rows(A, B, D, sample_rows(M, 64))
    assert frob <= 1e-3
    full = [torch.empty((M, N), dtype=torch.float16, device=f"cuda:{d}") for d in devices]
    b2g.allgather_rows(dD, full, devices=devices)
    for f in full:
        assert np.array_equal(to_host(f), D)


def test_cli_gpus_allgather():
    n = min(_ndev(), 2)
    out = subprocess.run([b2g.os.path.join(b2g.LIB_DIR, "gemm_bench"), "--gpus", str(n),
                          "--allgather", "--m", "1024", "--n", "768", "--k", "512", "--iters",
                          "5", "--warmup", "2", "--frob", "16", "--cpu", "64", "--json"],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "gather=OK" in out.stdout
    assert f"gpus={n}" in out.stdout


def _fused(A, B, bias, devices, *, D_pitch=None, **kw):
    """Run b2g_gemm_multi_allgather; returns the per-device D_full tensors."""
    M, N = A.shape[0], B.shape[0]
    dA, dB, dBias, _ = _panels(A, B, bias, devices)
    ld = D_pitch or N
    full = [torch.full((M, ld), float("nan"), dtype=torch.float16, device=f"cuda:{d}")[:, :N]
            for d in devices]
    b2g.gemm_multi_allgather(dA, dB, full, dBias if kw.get("epilogue") else None,
                             devices=devices, **kw)
    return full


def _separate(A, B, bias, devices, **kw):
    """The same product through b2g_gemm_multi (panels stacked on the host)."""
    dA, dB, dBias, dD = _panels(A, B, bias, devices)
    b2g.gemm_multi(dA, dB, dD, dBias if kw.get("epilogue") else None, M=A.shape[0],
                   devices=devices, **kw)
    return _assemble(dD)


@pytest.mark.parametrize("devices", [[0], [0, 0], [0, 0, 0, 0]])
@pytest.mark.parametrize("M,N,K", [(1024, 512, 512), (1000, 520, 200), (4096, 4096, 256),
                                   (520, 1024, 4096), (300, 136, 64)])
def test_fused_allgather_equals_separate(devices, M, N, K):
    """Every device's D_full from the fused kernel equals the separately computed panels bit
    for bit (same tiles, same k order), and agrees with the FP64 oracle."""
    A, B, bias = inputs(M, N, K, seed=M + 2 * N + K)
    full = _fused(A, B, bias, devices)
    ref = _separate(A, B, bias, devices)
    for f in full:
        assert np.array_equal(to_host(f), ref)
    frob, _ = check_rows(A, B, ref, sample_rows(M, 32))
    assert frob <= 1e-3


@pytest.mark.parametrize("kw", [dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.75),
                                dict(acc=b2g.ACC_F16), dict(tile=b2g.TILE_128x128),
                                dict(tile=b2g.TILE_256x512_2SM), dict(tile=b2g.TILE_128x64),
                                dict(tile=b2g.TILE_256x128_2SM), dict(b_layout=b2g.B_KN)])
def test_fused_allgather_modes(kw):
    devices = [0, 0]
    M, N, K = 1536, 1024, 576
    A, B, bias = inputs(M, N, K, seed=5, lo=-0.5, hi=0.5)
    if kw.get("b_layout") == b2g.B_KN:
        Bt = np.ascontiguousarray(B.T)
        dA, _, _, dD = _panels(A, B, bias, devices)
        dB = [to_dev(torch, Bt) for _ in devices]
        full = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _ in devices]
        b2g.gemm_multi_allgather(dA, dB, full, devices=devices, **kw)
        b2g.gemm_multi(dA, dB, dD, M=M, devices=devices, **kw)
        ref = _assemble(dD)
    else:
        full = _fused(A, B, bias, devices, **kw)
        ref = _separate(A, B, bias, devices, **kw)
    for f in full:
        assert np.array_equal(to_host(f), ref)


def test_fused_allgather_split_k_and_padded_pitch():
    """Small M per device with long K (split-K, the last split's reduction pushes the boxes)
    and D_full rows padded to a wider pitch."""
    devices = [0, 0]
    M, N, K = 256, 1024, 4096
    A, B, bias = inputs(M, N, K, seed=9)
    run(torch, A[:M // 2], B)  # one panel on this thread: the automatic choice splits K
    assert b2g.last_launch()["splits"] > 1
    full = _fused(A, B, bias, devices, D_pitch=N + 64)
    ref = _separate(A, B, bias, devices)
    for f in full:
        assert np.array_equal(to_host(f), ref)


def test_fused_allgather_k0_and_rejections():
    devices = [0, 0]
    M, N = 96, 64
    A = np.zeros((M, 0), np.uint16)
    B = np.zeros((N, 0), np.uint16)
    _, _, bias = inputs(M, N, 8)
    full = _fused(A, B, bias, devices, epilogue=b2g.EPI_BIAS_RELU)
    expect = b2g_f16(bias)
    for f in full:
        assert np.array_equal(to_host(f), np.broadcast_to(expect, (M, N)))
    A, B, bias = inputs(64, 60, 64)
    with pytest.raises(b2g.B2GError) as e:          # N % 8 != 0
        _fused(A, B, bias, devices)
    assert e.value.code == b2g.ERR_ALIGN
    A, B, bias = inputs(64, 64, 64)
    with pytest.raises(b2g.B2GError) as e:          # the swapped-operand kernel
        _fused(A, B, bias, devices, tile=b2g.TILE_SWAP_AB)
    assert e.value.code == b2g.ERR_UNSUPPORTED


def b2g_f16(bits):
    """FP16 bit patterns -> the same bit patterns after max(x, 0) in FP16 (as uint16)."""
    x = bits.view(np.float16).astype(np.float32)
    return np.maximum(x, 0).astype(np.float16).view(np.uint16)


@pytest.mark.skipif(_ndev() < 2, reason="needs two devices")
def test_two_devices_fused_allgather():
    devices = [0, 1]
    M, N, K = 4096, 2048, 1024
    A, B, bias = inputs(M, N, K, seed=13)
    full = _fused(A, B, bias, devices)
    ref = _separate(A, B, bias, devices)
    for f in full:
        assert np.array_equal(to_host(f), ref)
