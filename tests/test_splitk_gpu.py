"""Split-K GPU tests (b2g_gemm_splitk and the automatic split in b2g_gemm), against the FP64
oracle. The reference has no split-K; its skinny-M collapse (docs/RESULTS.md:249-265, M = 1..128
with N = K = 4096) is the case split-K exists for, so those shapes are checked here too."""
import numpy as np
import pytest

import b2g
import oracle as O
from helpers import check_rows, inputs, run, sample_rows, to_dev, to_host

pytestmark = pytest.mark.gpu

FROB_F32 = 1e-3
ELEM_F32 = 2 * 2.0 ** -11


@pytest.mark.parametrize("tile", [b2g.TILE_128x128, b2g.TILE_128x256, b2g.TILE_256x256_2SM,
                                  b2g.TILE_128x64, b2g.TILE_256x128_2SM])
@pytest.mark.parametrize("splits", [2, 3, 7, 16])
@pytest.mark.parametrize("fused", [False, True])
def test_forced_splits(cuda, tile, splits, fused):
    """Every tile kernel with S splits of K = 1000 (16 k-blocks, uneven shares, a ragged last
    k-block) on ragged M and N, with and without the fused alpha/bias/ReLU epilogue."""
    M, N, K = 300, 520, 1000
    A, B, bias = inputs(M, N, K, seed=31)
    lda = (K + 7) // 8 * 8
    kw = dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5) if fused else {}
    D = run(cuda, A, B, bias if fused else None, tile=tile, splits=splits, lda=lda, ldb=lda, **kw)
    launch = b2g.last_launch()
    assert launch["splits"] == splits and launch["units"] % splits == 0, launch
    frob, maxrel = check_rows(A, B, D, list(range(M)), bias=bias if fused else None,
                              alpha=kw.get("alpha", 1.0), epilogue=fused)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("splits", [2, 4])
def test_split_unaligned_output(cuda, splits):
    """Split-K with an output pitch TMA cannot store (ldd = N + 3): the last split writes
    its sums through the plain-store path."""
    M, N, K = 200, 300, 1024
    A, B, _ = inputs(M, N, K, seed=39)
    D = run(cuda, A, B, tile=b2g.TILE_128x128, splits=splits, ldd=N + 3)
    frob, maxrel = check_rows(A, B, D, list(range(M)))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


def test_split_result_is_deterministic_and_close_to_unsplit(cuda):
    """The last split sums partials in split order, so repeated runs are bit-identical; the
    split sum differs from the single-pass accumulation only by FP32 rounding."""
    M, N, K = 256, 768, 4096
    A, B, _ = inputs(M, N, K, seed=32)
    outs = [run(cuda, A, B, splits=8) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    one = run(cuda, A, B, splits=1)
    d = np.abs(O.f16_to_f32(outs[0]) - O.f16_to_f32(one))
    assert d.max() <= 2.0 ** -9 * max(1.0, np.abs(O.f16_to_f32(one)).max()), d.max()


@pytest.mark.parametrize("M,split,tile", [(1, 4, b2g.TILE_128x128), (8, 4, b2g.TILE_128x128),
                                          (32, 4, b2g.TILE_128x128), (128, 4, b2g.TILE_128x128),
                                          (256, 2, b2g.TILE_128x128),
                                          (512, 2, b2g.TILE_256x256_2SM),
                                          (1024, 1, b2g.TILE_256x256_2SM)])
def test_skinny_decode_auto_split(cuda, M, split, tile):
    """The reference's Phase 6 shapes (N = K = 4096): b2g_gemm splits K automatically when
    the tiles leave most SMs idle, each tile's splits forming one cluster reduced through
    distributed shared memory: 128 x 128 tiles for M <= 256, and at M = 512 two splits of
    256 x 256 pair tiles (clusters of two pairs); M = 1024 fills the GPU with pairs unsplit."""
    N = K = 4096
    A, B, _ = inputs(M, N, K, seed=33)
    D = run(cuda, A, B)
    launch = b2g.last_launch()
    assert (launch["tile"], launch["splits"]) == (tile, split), launch
    if split > 1:
        ctas = 2 if tile == b2g.TILE_256x256_2SM else 1
        assert launch["cluster"] == split * ctas and launch["grid"] == ctas * launch["units"]
    rows = sample_rows(M, 32)
    frob, maxrel = check_rows(A, B, D, rows)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


def test_split_rejections(cuda):
    A, B, _ = inputs(64, 64, 128, seed=34)
    with pytest.raises(b2g.B2GError) as e:
        run(cuda, A, B, acc=b2g.ACC_F16, splits=2)
    assert e.value.code == b2g.ERR_UNSUPPORTED
    with pytest.raises(b2g.B2GError) as e:
        run(cuda, A, B, splits=3)  # K = 128 has 2 k-blocks
    assert e.value.code == b2g.ERR_ARG
    with pytest.raises(b2g.B2GError) as e:
        run(cuda, A, B, splits=-1)
    assert e.value.code == b2g.ERR_ARG
    # FP16 accumulation never splits automatically
    A, B, _ = inputs(8, 512, 4096, seed=35, lo=-0.5, hi=0.5)
    run(cuda, A, B, acc=b2g.ACC_F16)
    assert b2g.last_launch()["splits"] == 1


def test_workspace_growth_and_streams(cuda):
    """Shapes that need a larger workspace in turn, then two streams at once: each stream
    has its own partials and counters, so concurrent split GEMMs do not interfere."""
    torch = cuda
    cases = [(64, 256, 512, 2), (128, 2048, 2048, 8), (256, 4096, 4096, 4), (64, 256, 512, 2)]
    for M, N, K, S in cases:
        A, B, _ = inputs(M, N, K, seed=36)
        D = run(cuda, A, B, splits=S)
        frob, maxrel = check_rows(A, B, D, sample_rows(M, 16))
        assert frob <= FROB_F32 and maxrel <= ELEM_F32, (M, N, K, S, frob, maxrel)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    jobs = []
    for seed, st in ((37, s1), (38, s2)):
        A, B, _ = inputs(128, 2048, 2048, seed=seed)
        dA, dB = to_dev(torch, A), to_dev(torch, B)
        dD = torch.empty(128, 2048, dtype=torch.float16, device="cuda")
        jobs.append((A, B, dA, dB, dD, st))
    torch.cuda.synchronize()
    for rep in range(4):
        for A, B, dA, dB, dD, st in jobs:
            b2g.gemm(dA, dB, dD, stream=st, splits=8)
    torch.cuda.synchronize()
    b2g.sync_status()
    for A, B, dA, dB, dD, st in jobs:
        frob, maxrel = check_rows(A, B, to_host(dD), sample_rows(128, 16))
        assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


def _split_pair(torch, A, B, bias, splits, tile, kw, lda):
    """The same split GEMM through b2g_gemm_splitk and b2g_gemm_splitk_noalloc (which always
    reduces through its static workspace); returns both outputs and the first's launch."""
    M, N = A.shape[0], B.shape[0]
    dA, dB = to_dev(torch, A, lda), to_dev(torch, B, lda)
    dbias = to_dev(torch, bias) if bias is not None else None
    outs, launch = [], None
    for fn in (b2g.gemm, b2g.gemm_noalloc):
        dD = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        fn(dA, dB, dD, dbias, tile=tile, splits=splits, **kw)
        b2g.sync_status()
        if launch is None:
            launch = b2g.last_launch()
        outs.append(to_host(dD))
    return outs, launch


PAIR_TILES = (b2g.TILE_256x256_2SM, b2g.TILE_256x128_2SM)


@pytest.mark.parametrize("tile,splits", [(b2g.TILE_128x128, 2), (b2g.TILE_128x128, 3),
                                         (b2g.TILE_128x128, 4), (b2g.TILE_128x128, 8),
                                         (b2g.TILE_128x64, 4), (b2g.TILE_128x64, 8),
                                         (b2g.TILE_128x256, 2), (b2g.TILE_128x256, 4),
                                         (b2g.TILE_256x256_2SM, 2), (b2g.TILE_256x256_2SM, 3),
                                         (b2g.TILE_256x256_2SM, 4), (b2g.TILE_256x128_2SM, 2),
                                         (b2g.TILE_256x128_2SM, 4)])
@pytest.mark.parametrize("fused", [False, True])
def test_cluster_reduction_matches_workspace(cuda, tile, splits, fused):
    """Split-K runs each tile's splits as one cluster (S CTAs, or S pairs of the 2-CTA
    kernel) and sums the partials in the shared memory of the owning CTA (st.async into its
    receive slots, which overlay its drained operand ring); the no-allocation entry point sums
    the same partials through its workspace. Same operations in the same split order:
    identical bits. Ragged M, N and K; uneven K shares."""
    M, N, K = 300, 520, 2000
    A, B, bias = inputs(M, N, K, seed=35)
    kw = dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5) if fused else {}
    (Dc, Dw), launch = _split_pair(cuda, A, B, bias if fused else None, splits, tile, kw, K)
    ctas = 2 if tile in PAIR_TILES else 1
    assert launch["cluster"] == splits * ctas and launch["grid"] == ctas * launch["units"], launch
    assert np.array_equal(Dc, Dw)
    frob, maxrel = check_rows(A, B, Dc, list(range(M)), bias=bias if fused else None,
                              alpha=kw.get("alpha", 1.0), epilogue=fused)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("M", [1, 8, 128])
def test_cluster_reduction_decode_is_deterministic(cuda, M):
    """The decode shapes (N = K = 4096, automatic split): three calls give the same bits, and
    the same bits as the workspace reduction of the no-allocation entry point."""
    torch = cuda
    A, B, _ = inputs(M, 4096, 4096, seed=36)
    outs = [run(torch, A, B) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    splits = b2g.last_launch()["splits"]
    (_, Dw), _ = _split_pair(torch, A, B, None, splits, b2g.TILE_128x128, {}, 4096)
    assert np.array_equal(outs[0], Dw)


def test_cluster_reduction_unaligned_output(cuda):
    """Owners of pieces write D through the plain-store path when TMA cannot (ldd = N + 3)."""
    M, N, K = 200, 300, 1024
    A, B, _ = inputs(M, N, K, seed=37)
    D = run(cuda, A, B, tile=b2g.TILE_128x128, splits=4, ldd=N + 3)
    assert b2g.last_launch()["cluster"] == 4
    frob, maxrel = check_rows(A, B, D, list(range(M)))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
