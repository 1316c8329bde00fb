"""GPU edge cases at the extremes of the size range, checked against the FP64 oracle on sampled
rows: an output with more than 2^31 elements (64-bit row offsets in every store path), very
long K (split-K and the cluster reduction over many k-blocks), a single output element with long
K, and very tall and very wide skinny outputs. The reference has no such tests (its sizes are
flags of one benchmark binary, src/gemm_bench.cu:698-745); these guard index arithmetic that
only large shapes reach."""
import numpy as np
import pytest

import b2g
import oracle as O
from helpers import inputs, to_dev, to_host

pytestmark = pytest.mark.gpu

FROB_F32 = 1e-3
ELEM_F32 = 2 * 2.0 ** -11


def _rows_of(torch, dD, rows):
    """Only the sampled rows come back to the host (the full D may be several GiB)."""
    idx = torch.tensor(rows, dtype=torch.long, device=dD.device)
    return to_host(dD.index_select(0, idx))


def _check(A, B, rows, got, tol_elem):
    R = np.concatenate([O.gemm_f64(A, B, 0, r, r + 1) for r in rows])
    frob = O.frobenius_rel(got, R)
    Df = O.f16_to_f32(got).astype(np.float64)
    assert np.all(np.isfinite(Df)), "unwritten or overflowed output elements"
    maxrel = float(np.max(np.abs(Df - R) / np.maximum(1.0, np.abs(R))))
    assert frob <= FROB_F32 and maxrel <= tol_elem, (frob, maxrel)
    return frob, maxrel


@pytest.mark.parametrize("tile", [b2g.TILE_AUTO, b2g.TILE_128x128])
def test_output_beyond_2_pow_31_elements(cuda, tile):
    """D of 65536 x 32800 FP16 (2.15e9 elements, 4.0 GiB): the rows past element 2^31 are
    written at the right place (TMA-store path, and the pair kernel's tail slices)."""
    torch = cuda
    M, N, K = 65536, 32800, 64
    A, B, _ = inputs(M, N, K, seed=91)
    dD = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    b2g.gemm(to_dev(torch, A), to_dev(torch, B), dD, tile=tile)
    b2g.sync_status()
    assert M * N > 2 ** 31
    first_big = (2 ** 31) // N  # first row holding an element past 2^31
    rows = [0, 1, first_big - 1, first_big, first_big + 1, M // 2, M - 2, M - 1]
    frob, maxrel = _check(A, B, rows, _rows_of(torch, dD, rows), ELEM_F32)
    print(f"65536 x 32800 x 64 (tile {b2g.last_launch()['tile']}): frob {frob:.2e} maxrel {maxrel:.2e}")


def test_unaligned_output_beyond_2_pow_31_elements(cuda):
    """The plain-store path (row pitch not a multiple of 8: no TMA store) past element 2^31."""
    torch = cuda
    M, N, K = 65537, 32769, 64
    A, B, _ = inputs(M, N, K, seed=92)
    buf = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    b2g.gemm(to_dev(torch, A), to_dev(torch, B), buf)
    b2g.sync_status()
    rows = [0, 2 ** 31 // N, 2 ** 31 // N + 1, M - 1]
    _check(A, B, rows, _rows_of(torch, buf, rows), ELEM_F32)


@pytest.mark.parametrize("M,N,K,splits", [(128, 256, 65536, 0), (256, 1024, 32768, 8),
                                          (64, 512, 131072, 4)])
def test_very_long_k(cuda, M, N, K, splits):
    """K up to 131072 (2048 k-blocks): the automatic split (cluster reduction) and forced
    splits. At this K the FP32 accumulation error itself (~sqrt(K) roundings of partial sums
    of ~sqrt(K / 9): ~1.3e-3 absolute at K = 65536) exceeds the FP16 output rounding and
    depends on the summation order, so the element-wise bound is twice cuBLAS's own error on
    the same rows (measured: 2.3e-3 vs 1.5e-3 at K = 65536); Frobenius stays <= 1e-3."""
    torch = cuda
    A, B, _ = inputs(M, N, K, seed=93, lo=-1.0, hi=1.0)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dD = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    b2g.gemm(dA, dB, dD, splits=splits)
    b2g.sync_status()
    launch = b2g.last_launch()
    rows = list(range(0, M, max(1, M // 16))) + [M - 1]
    ref = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    b2g.cublas_gemm(dA, dB, ref)
    b2g.sync_status()
    R = np.concatenate([O.gemm_f64(A, B, 0, r, r + 1) for r in rows])
    cub = to_host(ref)[rows]
    cub_err = float(np.max(np.abs(O.f16_to_f32(cub) - R) / np.maximum(1.0, np.abs(R))))
    frob, maxrel = _check(A, B, rows, to_host(dD)[rows], max(ELEM_F32, 2.0 * cub_err))
    print(f"{M}x{N}x{K}: {launch}, frob {frob:.2e} maxrel {maxrel:.2e} (cuBLAS {cub_err:.2e})")
    assert launch["splits"] > 1


def test_single_element_long_k(cuda):
    """M = N = 1, K = 65536: one output element, every k-block split across a cluster."""
    torch = cuda
    A, B, _ = inputs(1, 1, 65536, seed=94, lo=-0.25, hi=0.25)
    dD = torch.full((1, 1), float("nan"), dtype=torch.float16, device="cuda")
    b2g.gemm(to_dev(torch, A), to_dev(torch, B), dD)
    b2g.sync_status()
    R = O.gemm_f64(A, B)
    got = O.f16_to_f32(to_host(dD)).astype(np.float64)
    assert abs(got[0, 0] - R[0, 0]) <= max(1.0, abs(R[0, 0])) * 2.0 ** -10


@pytest.mark.parametrize("shape", [(262144, 64, 128), (64, 262144, 128)])
def test_tall_and_wide_skinny_outputs(cuda, shape):
    """A 262144-row and a 262144-column output with short K: many tiles along one axis."""
    torch = cuda
    M, N, K = shape
    A, B, _ = inputs(M, N, K, seed=95)
    dD = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    b2g.gemm(to_dev(torch, A), to_dev(torch, B), dD)
    b2g.sync_status()
    rows = [0, M // 3, M - 1] if M > 64 else list(range(M))
    _check(A, B, rows, _rows_of(torch, dD, rows), ELEM_F32)
