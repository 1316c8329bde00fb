"""GPU parity tests of the sm_100a GEMM, through the C-ABI, against the CPU oracle and the
reference's own sm_89 kernel (compiled from its source, JIT-run on the B200).

Tolerances (from the north star): relative Frobenius error vs FP64 <= 1e-3 for FP32
accumulation and <= 5e-3 for FP16 accumulation; the reference's own OK threshold on
max |x - y| / max(1, |y|) is 3e-2 (src/gemm_bench.cu:851, :861).
"""
import ctypes as C

import numpy as np
import pytest

import b2g
import oracle as O
from helpers import check_rows, inputs, run, sample_rows, to_dev, to_host

pytestmark = pytest.mark.gpu

FROB_F32 = 1e-3
FROB_F16 = 5e-3
REF_OK = 3e-2
# FP32 accumulation, FP16 output: the output rounding alone is up to 2^-11 relative; allow
# two half-ulps element-wise for accumulation-order differences
ELEM_F32 = 2 * 2.0 ** -11


def test_config1_512_elementwise_vs_fp32_triple_loop(cuda):
    """512^3, seed 0, U[-1,1], FP32 acc, element-wise vs FP32 loop."""
    A, B, _ = inputs(512, 512, 512, seed=0)
    D = run(cuda, A, B)
    R32 = O.gemm_f32_naive(A, B)
    Df = O.f16_to_f32(D)
    rel = np.abs(Df - R32) / np.maximum(1.0, np.abs(R32))
    assert rel.max() <= ELEM_F32, rel.max()
    assert O.frobenius_rel(D, O.gemm_f64(A, B)) <= FROB_F32


@pytest.mark.parametrize("tile", [b2g.TILE_128x128, b2g.TILE_128x256, b2g.TILE_256x256_2SM,
                                  b2g.TILE_128x64, b2g.TILE_256x512_2SM,
                                  b2g.TILE_256x128_2SM])
@pytest.mark.parametrize("shape", [(1, 1, 8), (1, 1, 1), (7, 9, 13), (128, 128, 64),
                                   (129, 257, 72), (300, 200, 100), (256, 512, 1000),
                                   (1000, 33, 64), (64, 640, 4096)])
def test_shapes_small(cuda, tile, shape):
    M, N, K = shape
    A, B, _ = inputs(M, N, K, seed=11)
    lda = (K + 7) // 8 * 8
    D = run(cuda, A, B, tile=tile, lda=lda, ldb=lda)
    frob, maxrel = check_rows(A, B, D, list(range(M)))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("tile", [b2g.TILE_128x128, b2g.TILE_128x256, b2g.TILE_256x256_2SM,
                                  b2g.TILE_128x64, b2g.TILE_256x512_2SM,
                                  b2g.TILE_256x128_2SM])
@pytest.mark.parametrize("stages", [2, 3, 4, 0])
@pytest.mark.parametrize("group", [1, 2, 8])
def test_tiles_stages_groups(cuda, tile, stages, group):
    A, B, _ = inputs(1024, 768, 320, seed=3)
    D = run(cuda, A, B, tile=tile, stages=stages, group=group)
    frob, maxrel = check_rows(A, B, D, sample_rows(1024, 96))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("shape", [(1024, 1024, 512), (300, 520, 200), (4096, 4096, 256),
                                   (2304, 4352, 128), (512, 300, 64)])
def test_pair_tail_slices(cuda, shape):
    """2-CTA kernel shapes whose last partial wave is cut into 128- or 64-column slices
    (including slices that lie wholly beyond N)."""
    M, N, K = shape
    A, B, _ = inputs(M, N, K, seed=13)
    D = run(cuda, A, B, tile=b2g.TILE_256x256_2SM)
    frob, maxrel = check_rows(A, B, D, sample_rows(M, 128))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("tile", [b2g.TILE_128x128, b2g.TILE_128x256, b2g.TILE_256x256_2SM,
                                  b2g.TILE_128x64, b2g.TILE_256x512_2SM,
                                  b2g.TILE_256x128_2SM])
@pytest.mark.parametrize("K,warps", [(1024, 8), (1088, 4), (64, 8)])
@pytest.mark.parametrize("mode", ["plain", "fused", "f16acc"])
@pytest.mark.parametrize("MN", [(640, 704), (2560, 2304)])
def test_epilogue_warps_by_k(cuda, tile, K, warps, mode, MN):
    """Without split-K, K <= 1024 launches 8 epilogue warps (two per TMEM lane quarter,
    alternate 64-column chunks, one staging box each) and longer K launches 4 (two boxes
    each), unless every CTA (pair) has a single tile, which takes 4 (no next mainloop to keep
    up with); all give the same result in every epilogue mode, including the tail slices of
    the 2-CTA kernel (640 x 704: one tile per CTA; 2560 x 2304: more tiles than CTAs)."""
    M, N = MN
    A, B, bias = inputs(M, N, K, seed=21, lo=-0.5, hi=0.5)
    kw = {}
    if mode == "fused":
        kw = dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.75)
    elif mode == "f16acc":
        kw = dict(acc=b2g.ACC_F16)
    D = run(cuda, A, B, bias if mode == "fused" else None, tile=tile, splits=1, **kw)
    launch = b2g.last_launch()
    ctas = 2 if tile in (b2g.TILE_256x256_2SM, b2g.TILE_256x512_2SM, b2g.TILE_256x128_2SM) else 1
    if tile == b2g.TILE_256x512_2SM:
        warps = 8  # always: the next tile's half-1 MMAs wait for this epilogue
    elif launch["units"] * ctas <= launch["grid"]:
        warps = 4  # one tile per CTA (pair)
    assert launch["threads"] == 64 + 32 * warps, launch
    assert launch["tile"] == tile
    rows = sample_rows(M, 96)
    frob, maxrel = check_rows(A, B, D, rows, bias=bias if mode == "fused" else None,
                              alpha=kw.get("alpha", 1.0), epilogue=mode == "fused")
    tol = FROB_F16 if mode == "f16acc" else FROB_F32
    assert frob <= tol, (frob, maxrel)
    if mode != "f16acc":
        assert maxrel <= ELEM_F32, (frob, maxrel)


def test_kernel_clock_telemetry(cuda):
    A, B, _ = inputs(1024, 1024, 1024, seed=14)
    run(cuda, A, B)
    mhz, us = b2g.kernel_clock()
    print(f"kernel clock {mhz:.0f} MHz over {us:.1f} us")
    assert 500 < mhz < 2500 and us > 0


def test_headline_4096_fp32acc(cuda):
    """4096^3, seed 1, U[-1,1], FP32 accumulation."""
    A, B, _ = inputs(4096, 4096, 4096, seed=1)
    D = run(cuda, A, B)
    frob, maxrel = check_rows(A, B, D, sample_rows(4096, 64))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
    w, _, _ = O.spot_check(A, B, D, samples=512)
    assert w < REF_OK and w <= ELEM_F32, w


def test_f16acc_4096(cuda):
    """4096^3, seed 2, U[-0.5,0.5], FP16 accumulation."""
    A, B, _ = inputs(4096, 4096, 4096, seed=2, lo=-0.5, hi=0.5)
    D = run(cuda, A, B, acc=b2g.ACC_F16)
    frob, maxrel = check_rows(A, B, D, sample_rows(4096, 64))
    print(f"f16acc 4096^3: frob {frob:.3e} maxrel {maxrel:.3e}")
    assert frob <= FROB_F16, frob


@pytest.mark.parametrize("shape", [(4095, 4095, 4095), (5000, 3000, 2000)])
def test_ragged_baseline_shapes(cuda, shape):
    """BASELINE config 4 ragged shapes; K not a multiple of 8 needs a padded lda/ldb."""
    M, N, K = shape
    A, B, _ = inputs(M, N, K, seed=4)
    lda = (K + 7) // 8 * 8
    D = run(cuda, A, B, lda=lda, ldb=lda)
    frob, maxrel = check_rows(A, B, D, sample_rows(M, 48))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("shape", [(16384, 16384, 256), (256, 16384, 16384)])
def test_skinny_baseline_shapes(cuda, shape):
    """BASELINE config 4 skinny shapes. At K = 16384 the FP32 accumulation error itself
    (~sqrt(K) roundings of partial sums ~|D|) exceeds two FP16 half-ulps for elements
    near 1, so the element-wise bound there is cuBLAS's own error on the same rows."""
    torch = cuda
    M, N, K = shape
    A, B, _ = inputs(M, N, K, seed=5)
    D = run(cuda, A, B)
    rows = sample_rows(M, 16)
    frob, maxrel = check_rows(A, B, D, rows)
    assert frob <= FROB_F32, frob
    dD = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    b2g.cublas_gemm(to_dev(torch, A), to_dev(torch, B), dD)
    b2g.sync_status()
    _, cublas_maxrel = check_rows(A, B, to_host(dD), rows)
    print(f"{shape}: frob {frob:.3e} maxrel {maxrel:.3e} (cuBLAS maxrel {cublas_maxrel:.3e})")
    assert maxrel <= max(ELEM_F32, 1.5 * cublas_maxrel), (maxrel, cublas_maxrel)


@pytest.mark.parametrize("alpha", [1.0, 0.5])
@pytest.mark.parametrize("with_bias", [True, False])
def test_fused_epilogue(cuda, alpha, with_bias):
    A, B, bias = inputs(384, 320, 192, seed=6)
    bias = bias if with_bias else None
    D = run(cuda, A, B, bias, epilogue=b2g.EPI_BIAS_RELU, alpha=alpha)
    frob, maxrel = check_rows(A, B, D, list(range(384)), bias=bias, alpha=alpha, epilogue=True)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
    assert (O.f16_to_f32(D) >= 0).all()


def test_unaligned_output_ld(cuda):
    A, B, _ = inputs(200, 300, 64, seed=7)
    D = run(cuda, A, B, ldd=301)
    frob, maxrel = check_rows(A, B, D, list(range(200)))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32


@pytest.mark.parametrize("tile", [b2g.TILE_128x128, b2g.TILE_256x256_2SM])
@pytest.mark.parametrize("fused", [False, True])
def test_unaligned_output_base(cuda, tile, fused):
    """D starting 2 bytes past a 16-byte boundary (no TMA store possible): the staging box is
    written out with plain row stores; neighbours outside D stay untouched."""
    torch = cuda
    M, N, K = 333, 520, 192
    A, B, bias = inputs(M, N, K, seed=8)
    buf = torch.full((M, N + 8), float("nan"), dtype=torch.float16, device="cuda")
    dD = buf[:, 1:N + 1]
    kw = dict(epilogue=b2g.EPI_BIAS_RELU, alpha=1.5) if fused else {}
    b2g.gemm(to_dev(torch, A), to_dev(torch, B), dD, to_dev(torch, bias) if fused else None,
             tile=tile, **kw)
    b2g.sync_status()
    out = to_host(buf)
    frob, maxrel = check_rows(A, B, np.ascontiguousarray(out[:, 1:N + 1]), list(range(M)),
                              bias=bias if fused else None, alpha=kw.get("alpha", 1.0),
                              epilogue=fused)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
    assert np.isnan(O.f16_to_f32(out[:, 0])).all() and np.isnan(O.f16_to_f32(out[:, N + 1:])).all()


def test_k_zero_and_empty(cuda):
    torch = cuda
    A = torch.zeros((64, 0), dtype=torch.float16, device="cuda")
    B = torch.zeros((48, 0), dtype=torch.float16, device="cuda")
    D = torch.full((64, 48), 7.0, dtype=torch.float16, device="cuda")
    b2g.gemm(A, B, D)
    b2g.sync_status()
    assert (D == 0).all()
    bias = torch.linspace(-1, 1, 48, dtype=torch.float16, device="cuda")
    b2g.gemm(A, B, D, bias, epilogue=b2g.EPI_BIAS_RELU)
    b2g.sync_status()
    assert torch.equal(D, torch.relu(bias)[None, :].expand(64, 48))
    E = torch.full((0, 48), 1.0, dtype=torch.float16, device="cuda")
    b2g.gemm(torch.zeros((0, 8), dtype=torch.float16, device="cuda"),
             torch.zeros((48, 8), dtype=torch.float16, device="cuda"), E)
    b2g.sync_status()


def test_rejects_unaligned_inputs(cuda):
    torch = cuda
    A = torch.zeros((64, 100), dtype=torch.float16, device="cuda")
    B = torch.zeros((64, 100), dtype=torch.float16, device="cuda")
    D = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(b2g.B2GError) as e:
        b2g.gemm(A, B, D)  # lda = 100 is not a multiple of 8
    assert e.value.code == b2g.ERR_ALIGN
    buf = torch.zeros(64 * 104 + 8, dtype=torch.float16, device="cuda")
    with pytest.raises(b2g.B2GError) as e:
        b2g.gemm_raw(buf.data_ptr() + 2, B.data_ptr(), D.data_ptr(), None, 64, 64, 96, 104,
                     100, 64)
    assert e.value.code in (b2g.ERR_ALIGN,)
    b2g.sync_status()


def test_unfused_bias_relu_kernel(cuda):
    torch = cuda
    A, B, bias = inputs(130, 70, 1, seed=8)
    D = O.f32_to_f16(O.f16_to_f32(A)[:, :1] * np.linspace(-3, 3, 70, dtype=np.float32)[None, :])
    dD = to_dev(torch, D)
    b2g.bias_relu(dD, to_dev(torch, bias), alpha=0.75)
    b2g.sync_status()
    assert np.array_equal(to_host(dD), O.bias_relu(D, bias, 0.75))


def test_max_rel_diff_kernel(cuda):
    torch = cuda
    x = O.fill_uniform((1000, 37), 9, 0, -4, 4)
    y = O.fill_uniform((1000, 37), 9, 1, -4, 4)
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    b2g.max_rel_diff(to_dev(torch, x), to_dev(torch, y), out)
    b2g.sync_status()
    assert out.item() == O.max_rel_diff(x, y)


def test_cublas_column(cuda):
    torch = cuda
    A, B, _ = inputs(512, 384, 256, seed=10)
    dD = torch.zeros((512, 384), dtype=torch.float16, device="cuda")
    b2g.cublas_gemm(to_dev(torch, A), to_dev(torch, B), dD)
    b2g.sync_status()
    frob, maxrel = check_rows(A, B, to_host(dD), list(range(512)))
    assert frob <= FROB_F32 and maxrel < REF_OK


def test_selftest_wait_timeout_then_gemm_still_works(cuda):
    """A bounded device wait that nothing satisfies returns an error; the context lives."""
    assert b2g.selftest_wait_timeout(20000) == b2g.ERR_TIMEOUT
    assert "selftest" in b2g.last_error()
    b2g.sync_status()  # status word was cleared
    A, B, _ = inputs(256, 256, 128, seed=12)
    D = run(cuda, A, B)
    frob, _ = check_rows(A, B, D, list(range(256)))
    assert frob <= FROB_F32


def test_probe_tcgen05(cuda):
    rates = {}
    for kind in (0, 1, 2, 3):
        fl, cyc = b2g.probe_tcgen05(kind, 1, 256, 2048)
        rates[kind] = fl
        print(f"probe kind {kind} ({b2g.PROBE_KINDS[kind]}): {fl:.1f} FLOP/clk/SM, {cyc} cycles")
        assert cyc > 0
    # dense kind::f16 on one SM: 128x256x16 per MMA; nominal 8192 FLOP/clk/SM
    assert 2000 < rates[0] < 9000
    assert rates[2] > rates[0] * 1.5  # 8-bit kinds issue at least ~2x the 16-bit rate


def test_probe_tcgen05_pair(cuda):
    """cta_group::2: the pair MMA (UMMA M = 256 over two SMs) of the 2-CTA GEMM kernels,
    FLOP per clock per SM comparable with the one-SM rate, for every kind."""
    one, _ = b2g.probe_tcgen05(0, 1, 256, 2048)
    for kind in (0, 1, 2, 3):
        fl, cyc = b2g.probe_tcgen05(kind, 2, 256, 2048)
        print(f"pair probe kind {kind} ({b2g.PROBE_KINDS[kind]}): {fl:.1f} FLOP/clk/SM, "
              f"{cyc} cycles (one-SM kind 0: {one:.1f})")
        assert cyc > 0
        lo = 0.8 * one * (2 if kind >= 2 else 1)
        assert lo < fl < 1.25 * one * (2 if kind >= 2 else 1), (kind, fl, one)
    with pytest.raises(b2g.B2GError) as e:
        b2g.probe_tcgen05(0, 3, 256, 16)
    assert e.value.code == b2g.ERR_ARG


def test_probe_hbm(cuda):
    torch = cuda
    n = 1 << 30
    src = torch.empty(n, dtype=torch.uint8, device="cuda")
    dst = torch.empty(n, dtype=torch.uint8, device="cuda")
    gbs = b2g.probe_hbm(src, dst, n, reps=10)
    print(f"hbm copy {gbs:.1f} GB/s")
    assert gbs > 2000


@pytest.mark.parametrize("tile", [b2g.TILE_128x128, b2g.TILE_128x256, b2g.TILE_256x256_2SM,
                                  b2g.TILE_128x64, b2g.TILE_256x512_2SM,
                                  b2g.TILE_256x128_2SM])
@pytest.mark.parametrize("shape", [(384, 512, 256), (300, 520, 200), (1000, 64, 1000),
                                   (129, 1000, 72), (2304, 4352, 128)])
def test_b_kn_layout(cuda, tile, shape):
    """B stored K x N (b_layout B_KN, MN-major UMMA operand): every tile kernel, ragged M, N
    and K, and 2-CTA shapes whose last wave is cut into 128-column slices."""
    M, N, K = shape
    A, Bnk, _ = inputs(M, N, K, seed=51)
    Bkn = np.ascontiguousarray(Bnk.T)  # K x N
    ldb = (N + 7) // 8 * 8
    lda = (K + 7) // 8 * 8
    D = run(cuda, A, Bkn, tile=tile, b_layout=b2g.B_KN, lda=lda, ldb=ldb)
    frob, maxrel = check_rows(A, Bkn, D, sample_rows(M, 96), b_layout=1)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
    # identical to the N x K layout of the same matrix (same MMAs, same order)
    Dnk = run(cuda, A, Bnk, tile=tile, lda=lda, ldb=lda)
    assert np.array_equal(D, Dnk)


@pytest.mark.parametrize("mode", ["fused", "f16acc", "split"])
def test_b_kn_layout_modes(cuda, mode):
    M, N, K = 256, 768, 2048
    A, Bnk, bias = inputs(M, N, K, seed=52, lo=-0.5, hi=0.5)
    Bkn = np.ascontiguousarray(Bnk.T)
    kw = {"fused": dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5), "f16acc": dict(acc=b2g.ACC_F16),
          "split": dict(splits=4, tile=b2g.TILE_128x128)}[mode]
    b = bias if mode == "fused" else None
    D = run(cuda, A, Bkn, b, b_layout=b2g.B_KN, **kw)
    Dnk = run(cuda, A, Bnk, b, **kw)
    assert np.array_equal(D, Dnk)
    frob, maxrel = check_rows(A, Bkn, D, sample_rows(M, 64), bias=b, alpha=kw.get("alpha", 1.0),
                              epilogue=mode == "fused", b_layout=1)
    assert frob <= (FROB_F16 if mode == "f16acc" else FROB_F32), (frob, maxrel)


@pytest.mark.parametrize("shape,tile,splits", [
    ((1024, 1024, 1024), b2g.TILE_128x64, 1),      # sparse 128x128 tiles, short K
    ((512, 512, 512), b2g.TILE_128x64, 1),
    ((1024, 1024, 4096), b2g.TILE_128x128, 2),     # long K: split instead
    ((128, 4096, 4096), b2g.TILE_128x128, 4),      # decode-shaped
    ((512, 4096, 4096), b2g.TILE_256x256_2SM, 2),  # half-filled pairs: 2 K splits, one cluster
    ((2048, 1024, 1024), b2g.TILE_128x128, 1),     # 128 tiles: a full wave of 128x128
    ((4096, 4096, 4096), b2g.TILE_256x256_2SM, 1),  # the headline shape
    ((8192, 8192, 8192), b2g.TILE_256x512_2SM, 1),  # long K, >= 4 waves of 256 x 512
    ((16, 16384, 1024), b2g.TILE_SWAP_AB, 1),       # tiny M, wide N: swapped operands
    ((16, 4096, 4096), b2g.TILE_128x128, 4),        # tiny M, N = 4096: split-K instead
])
def test_auto_tile_choice(cuda, shape, tile, splits):
    """The automatic configuration (tile kernel and split factor) for representative shapes,
    each choice measured fastest on B200; the result is checked as well."""
    M, N, K = shape
    A, B, _ = inputs(M, N, K, seed=61)
    D = run(cuda, A, B)
    launch = b2g.last_launch()
    assert (launch["tile"], launch["splits"]) == (tile, splits), launch
    frob, maxrel = check_rows(A, B, D, sample_rows(M, 32))
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)


@pytest.mark.parametrize("shape,kw,variant", [
    ((512, 512, 512), {}, "plain"),                                   # 1-CTA, no split
    ((2048, 2048, 2048), {}, "plain"),                                # pair tiles
    ((2048, 1536, 1024), dict(tile=b2g.TILE_256x512_2SM), "plain"),  # wide pair tiles
    ((512, 512, 512), dict(acc=b2g.ACC_F16), "general"),
    ((512, 512, 512), dict(epilogue=b2g.EPI_BIAS_RELU, alpha=0.5), "general"),
    ((128, 4096, 4096), {}, "csplit"),                                # decode: split in a cluster
    ((512, 4096, 4096), {}, "csplit"),                                # pairs split in a cluster
    ((1024, 1024, 1024), dict(b_layout=b2g.B_KN, tile=b2g.TILE_256x256_2SM), "general"),
    ((1024, 1024, 1024), dict(b_layout=b2g.B_KN, tile=b2g.TILE_128x128), "plain"),
])
def test_kernel_variant_by_mode(cuda, shape, kw, variant):
    """Each tile kernel is compiled as a plain-path form (no split-K, FP32 accumulation, plain
    store, no peers; the pair kernel's also N x K B only), a cluster split-K form and a general
    one; the launch record names the form that ran, and each gives correct results."""
    M, N, K = shape
    A, B, bias = inputs(M, N, K, seed=81, lo=-0.5, hi=0.5)
    b_layout = kw.get("b_layout", b2g.B_NK)
    Bx = np.ascontiguousarray(B.T) if b_layout == b2g.B_KN else B
    epi = kw.get("epilogue", b2g.EPI_NONE) != b2g.EPI_NONE
    D = run(cuda, A, Bx, bias if epi else None, **kw)
    launch = b2g.last_launch()
    assert launch["variant"] == variant, launch
    frob, _ = check_rows(A, Bx, D, sample_rows(M, 32), bias=bias if epi else None,
                         alpha=kw.get("alpha", 1.0), epilogue=epi, b_layout=b_layout)
    assert frob <= (FROB_F16 if kw.get("acc") == b2g.ACC_F16 else FROB_F32), frob


@pytest.mark.parametrize("shape", [(2304, 4352, 320), (1024, 1536, 1000), (4096, 3000, 512),
                                   (520, 700, 128)])
@pytest.mark.parametrize("b_layout", [b2g.B_NK, b2g.B_KN])
def test_wide_pair_tile(cuda, shape, b_layout):
    """256 x 512 pair tiles (tile 4): two 256-column accumulator halves released separately
    to the next tile, with tail slices of 256 and 128 columns, ragged N, both B layouts; the
    output is bit-identical to the 256 x 256 kernel's (same K order per element)."""
    M, N, K = shape
    A, Bnk, _ = inputs(M, N, K, seed=71)
    lda = (K + 7) // 8 * 8
    if b_layout == b2g.B_KN:
        B = np.ascontiguousarray(Bnk.T)
        ldb = (N + 7) // 8 * 8
    else:
        B, ldb = Bnk, lda
    D = run(cuda, A, B, tile=b2g.TILE_256x512_2SM, b_layout=b_layout, lda=lda, ldb=ldb)
    assert b2g.last_launch()["tile"] == b2g.TILE_256x512_2SM
    frob, maxrel = check_rows(A, B, D, sample_rows(M, 96), b_layout=b_layout)
    assert frob <= FROB_F32 and maxrel <= ELEM_F32, (frob, maxrel)
    D2 = run(cuda, A, B, tile=b2g.TILE_256x256_2SM, b_layout=b_layout, lda=lda, ldb=ldb)
    assert np.array_equal(D, D2)


def test_wide_pair_tile_rejects_split(cuda):
    A, B, _ = inputs(512, 512, 1024, seed=72)
    with pytest.raises(b2g.B2GError) as e:
        run(cuda, A, B, tile=b2g.TILE_256x512_2SM, splits=2)
    assert e.value.code == b2g.ERR_UNSUPPORTED
