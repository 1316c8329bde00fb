"""Swapped-operand kernel (tile B2G_TILE_SWAP_AB) for decode-shaped GEMMs, against the FP64
oracle: B's rows on the UMMA's 128-row side, the small M as UMMA N (MT = 16, 32 or 64)."""
import numpy as np
import pytest

import b2g
import oracle as O
from helpers import check_rows, inputs, run, sample_rows

pytestmark = pytest.mark.gpu

FROB_F32 = 1e-3
FROB_F16 = 5e-3
ELEM_F32 = 2 * 2.0 ** -11


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64, 100, 256])
@pytest.mark.parametrize("N,K", [(4096, 4096), (1000, 100), (130, 1000)])
def test_swap_shapes(cuda, M, N, K):
    A, B, _ = inputs(M, N, K, seed=81)
    lda = (K + 7) // 8 * 8
    D = run(cuda, A, B, tile=b2g.TILE_SWAP_AB, lda=lda, ldb=lda)
    assert b2g.last_launch()["tile"] == b2g.TILE_SWAP_AB
    frob, maxrel = check_rows(A, B, D, sample_rows(M, 24))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("mode", ["fused", "f16acc", "unaligned_d"])
def test_swap_modes(cuda, mode):
    M, N, K = 40, 777, 2048
    A, B, bias = inputs(M, N, K, seed=82, lo=-0.5, hi=0.5)
    kw = {"fused": dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5), "f16acc": dict(acc=b2g.ACC_F16),
          "unaligned_d": dict(ldd=N + 3)}[mode]
    b = bias if mode == "fused" else None
    D = run(cuda, A, B, b, tile=b2g.TILE_SWAP_AB, **kw)
    frob, maxrel = check_rows(A, B, D, list(range(M)), bias=b, alpha=kw.get("alpha", 1.0),
                              epilogue=mode == "fused")
    assert frob <= (FROB_F16 if mode == "f16acc" else FROB_F32), (frob, maxrel)
    if mode != "f16acc":
        assert maxrel <= ELEM_F32, (frob, maxrel)
    if mode == "fused":
        assert (O.f16_to_f32(D) >= 0).all()


def test_swap_matches_normal_tiles_bitwise(cuda):
    """Same k order per output element as the 128 x 128 kernel without split-K."""
    M, N, K = 64, 1024, 3000
    A, B, _ = inputs(M, N, K, seed=83)
    lda = (K + 7) // 8 * 8
    D1 = run(cuda, A, B, tile=b2g.TILE_SWAP_AB, lda=lda, ldb=lda)
    D2 = run(cuda, A, B, tile=b2g.TILE_128x128, splits=1, lda=lda, ldb=lda)
    assert np.array_equal(D1, D2)


def test_swap_rejections(cuda):
    A, B, _ = inputs(8, 256, 256, seed=84)
    with pytest.raises(b2g.B2GError) as e:
        run(cuda, A, np.ascontiguousarray(B.T), tile=b2g.TILE_SWAP_AB, b_layout=b2g.B_KN)
    assert e.value.code == b2g.ERR_UNSUPPORTED
    with pytest.raises(b2g.B2GError) as e:
        run(cuda, A, B, tile=b2g.TILE_SWAP_AB, splits=2)
    assert e.value.code == b2g.ERR_UNSUPPORTED
