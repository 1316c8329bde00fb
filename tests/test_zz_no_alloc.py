"""b2g_gemm_splitk_noalloc (split-K scratch from a static device array, no allocation)
against the existing entry point b2g_gemm_splitk, on the GPU. Named to be collected last,
after every other test has used the library on the device; it also passes when run alone."""
import numpy as np
import pytest

import b2g
from helpers import check_rows, inputs, sample_rows, to_dev, to_host

pytestmark = pytest.mark.gpu

FROB_F32 = 1e-3
ELEM_F32 = 2 * 2.0 ** -11


def _pair(torch, M, N, K, seed, splits, tile=b2g.TILE_AUTO, fused=False):
    """Two calls in a row through each entry point on the same inputs; returns the four
    outputs (host) and the inputs."""
    A, B, bias = inputs(M, N, K, seed=seed)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dbias = to_dev(torch, bias) if fused else None
    kw = dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5) if fused else {}
    outs = []
    for fn in (lambda d: b2g.gemm(dA, dB, d, dbias, tile=tile, splits=splits, **kw),
               lambda d: b2g.gemm_noalloc(dA, dB, d, dbias, tile=tile, splits=splits, **kw)):
        for _ in range(2):
            dD = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            fn(dD)
            b2g.sync_status()
            outs.append(to_host(dD))
    return outs, (A, B, bias, kw)


@pytest.mark.parametrize("M,N,K,splits,tile", [
    (128, 4096, 4096, 4, b2g.TILE_128x128),    # decode-shaped, the automatic choice's case
    (1, 2048, 4096, 0, b2g.TILE_AUTO),         # automatic split
    (300, 520, 1000, 3, b2g.TILE_256x256_2SM),  # 2-CTA pair tiles, ragged edges
    (512, 512, 512, 1, b2g.TILE_AUTO),         # no split: no scratch used at all
])
def test_noalloc_matches_existing_entry_point(cuda, M, N, K, splits, tile):
    (e1, e2, n1, n2), (A, B, _, _) = _pair(cuda, M, N, K, 41, splits, tile)
    # the split sum is in fixed split order: both entry points give the same bits, every call
    assert np.array_equal(e1, e2) and np.array_equal(n1, n2) and np.array_equal(e1, n1)
    frob, maxrel = check_rows(A, B, n2, sample_rows(M, 32))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


def test_noalloc_fused_epilogue(cuda):
    (e1, e2, n1, n2), (A, B, bias, kw) = _pair(cuda, 64, 1024, 2048, 42, 4,
                                               b2g.TILE_128x128, fused=True)
    assert np.array_equal(e1, n1) and np.array_equal(n1, n2)
    frob, maxrel = check_rows(A, B, n1, list(range(64)), bias=bias, alpha=kw["alpha"],
                              epilogue=True)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


def test_noalloc_allocates_nothing(cuda):
    """No device memory changes hands: the CUDA free-memory figure is the same before and
    after split calls of a shape this process has not run before."""
    torch = cuda
    A, B, _ = inputs(96, 3072, 4096, seed=43)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dD = torch.empty((96, 3072), dtype=torch.float16, device="cuda")
    b2g.gemm_noalloc(dA, dB, dD, splits=4)  # first call: looks up the scratch address
    b2g.sync_status()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for s in (2, 3, 4):
        b2g.gemm_noalloc(dA, dB, dD, splits=s)
    b2g.sync_status()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    frob, maxrel = check_rows(A, B, to_host(dD), sample_rows(96, 16))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


def test_noalloc_rejects_oversize(cuda):
    """A split that needs more than the 16 MiB of static partials is refused with the sizes
    in the message, and launches nothing (D keeps its contents)."""
    torch = cuda
    M = N = 2048
    K = 4096
    A, B, _ = inputs(M, N, K, seed=44)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dD = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    with pytest.raises(b2g.B2GError) as e:  # 256 tiles x 16 splits x 64 KiB = 256 MiB
        b2g.gemm_noalloc(dA, dB, dD, tile=b2g.TILE_128x128, splits=16)
    assert e.value.code == b2g.ERR_ARG and "no-allocation scratch" in str(e.value)
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(dD)) == 0
    # the same shape without a split needs no scratch
    b2g.gemm_noalloc(dA, dB, dD, splits=1)
    b2g.sync_status()
    frob, _ = check_rows(A, B, to_host(dD), sample_rows(M, 8))
    assert frob <= FROB_F32
