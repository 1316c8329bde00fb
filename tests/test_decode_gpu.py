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


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (8, 4096, 4096), (17, 4096, 4096),
                                   (32, 4096, 4096), (5, 4100, 1000), (24, 2048, 130)])
def test_swap_narrow_form(cuda, M, N, K):
    """Decode shapes whose 128-row blocks of B would leave most SMs idle take the narrow form:
    ~N / SMs rows of B per CTA, several k-blocks per ring stage (one 3D load per operand and
    stage when K % 64 == 0), no split-K. Checked against the FP64 oracle on every row, and bit for bit against the
    128 x 128 tile kernel without split-K (same k order per element). Ragged N and K cover a
    partial last block of B rows and a short last ring stage."""
    A, B, _ = inputs(M, N, K, seed=85)
    lda = (K + 7) // 8 * 8
    D = run(cuda, A, B, tile=b2g.TILE_SWAP_AB, lda=lda, ldb=lda)
    launch = b2g.last_launch()
    assert launch["tile"] == b2g.TILE_SWAP_AB and launch["variant"] == "narrow", launch
    if N >= 4096:  # 32 rows of B per CTA (K % 64 == 0: 3D loads), else 28
        assert launch["grid"] == (128 if K % 64 == 0 else 147), launch
    frob, maxrel = check_rows(A, B, D, list(range(M)))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
    D2 = run(cuda, A, B, tile=b2g.TILE_128x128, splits=1, lda=lda, ldb=lda)
    assert np.array_equal(D, D2)


@pytest.mark.parametrize("mode", ["fused", "f16acc", "unaligned_d"])
def test_swap_narrow_modes(cuda, mode):
    """The narrow form with the fused epilogue, FP16 accumulation and an output pitch with
    no 16-byte alignment (N = K = 4096: 128 CTAs of 32 rows of B)."""
    M, N, K = 12, 4096, 4096
    A, B, bias = inputs(M, N, K, seed=86, lo=-0.5, hi=0.5)
    kw = {"fused": dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5), "f16acc": dict(acc=b2g.ACC_F16),
          "unaligned_d": dict(ldd=N + 3)}[mode]
    b = bias if mode == "fused" else None
    D = run(cuda, A, B, b, tile=b2g.TILE_SWAP_AB, **kw)
    assert b2g.last_launch()["variant"] == "narrow"
    frob, maxrel = check_rows(A, B, D, list(range(M)), bias=b, alpha=kw.get("alpha", 1.0),
                              epilogue=mode == "fused")
    assert frob <= (FROB_F16 if mode == "f16acc" else FROB_F32), (frob, maxrel)
    if mode != "f16acc":
        assert maxrel <= ELEM_F32, (frob, maxrel)


def test_swap_wide_form(cuda):
    """N wide enough for ~one 128-row block per SM keeps the 128-row form."""
    M, N, K = 16, 16384, 1024
    A, B, _ = inputs(M, N, K, seed=87)
    D = run(cuda, A, B, tile=b2g.TILE_SWAP_AB)
    launch = b2g.last_launch()
    assert launch["variant"] == "general" and launch["grid"] == 128, launch
    D2 = run(cuda, A, B, tile=b2g.TILE_128x128, splits=1)
    assert np.array_equal(D, D2)
