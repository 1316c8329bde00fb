"""GPU parity against the reference's OWN kernel and its published known answers.

The reference's gemm_kernel is compiled from its unmodified source (oracle/ref_shim.cu,
compute_89 PTX) and JIT-run on the B200 on the same inputs as ours. Known answers from the
reference's docs, with its LCG init (src/gemm_bench.cu:760-765) at 4096^3 and its
`--cpu 512` spot check (README.md:440):
  FP32 accumulate: 4.53e-04 (docs/RESULTS.md:396; 4.4e-04 .. 4.9e-04 at every shape, :624-627)
  FP16 accumulate: 3.78e-02 (docs/RESULTS.md:396, README.md:365)
"""
import numpy as np
import pytest

import b2g
import oracle as O
from helpers import inputs, run, to_dev, to_host

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")]

REF_OK = 3e-2
V_PLAIN, V_FUSED, V_F16ACC, V_K8 = 0, 1, 2, 3


def ref_gemm(torch, variant, A, B, bias=None, group=2, tile=3, stages=3, layout=2):
    M, K = A.shape
    N = B.shape[0]
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dbias = to_dev(torch, bias) if bias is not None else None
    dD = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    rc = O.ref().ref_gemm_launch(variant, dA.data_ptr(), dB.data_ptr(), dD.data_ptr(),
                                 None if dbias is None else dbias.data_ptr(), M, N, K, 1.0,
                                 group, tile, stages, layout,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0, f"reference kernel launch failed: cudaError {rc}"
    torch.cuda.synchronize()
    return to_host(dD)


@pytest.mark.parametrize("shape", [(512, 512, 512), (1024, 768, 256), (4096, 4096, 4096)])
def test_matches_reference_kernel(cuda, shape):
    M, N, K = shape
    A, B, _ = inputs(M, N, K, init="lcg")
    ours = run(cuda, A, B)
    theirs = ref_gemm(cuda, V_K8, A, B)
    d = O.max_rel_diff(ours, theirs)
    print(f"{shape}: max rel diff ours vs reference kernel {d:.3e}")
    assert d < REF_OK
    # both kernels round an FP32 accumulator to FP16: at most one FP16 ulp apart
    assert d <= 2 * 2.0 ** -11


def test_known_answer_fp32acc_4096(cuda):
    A, B, _ = inputs(4096, 4096, 4096, init="lcg")
    theirs = ref_gemm(cuda, V_K8, A, B)
    w_ref, m, n = O.spot_check(A, B, theirs, samples=512)
    print(f"reference kernel cpu=512 spot check: {w_ref:.3e} (worst m={m} n={n})")
    assert f"{w_ref:.2e}" == "4.53e-04"  # the reference's published figure, reproduced
    ours = run(cuda, A, B)
    w, m, n = O.spot_check(A, B, ours, samples=512)
    print(f"ours cpu=512 spot check: {w:.3e} (worst m={m} n={n})")
    assert 4.4e-4 <= w <= 4.9e-4 or w <= w_ref


def test_known_answer_f16acc_4096(cuda):
    A, B, _ = inputs(4096, 4096, 4096, init="lcg")
    theirs = ref_gemm(cuda, V_F16ACC, A, B)
    w_ref, _, _ = O.spot_check(A, B, theirs, samples=512)
    ours = run(cuda, A, B, acc=b2g.ACC_F16)
    w, _, _ = O.spot_check(A, B, ours, samples=512)
    print(f"f16 accumulate cpu=512: reference kernel {w_ref:.3e} (published 3.78e-02), ours {w:.3e}")
    assert 1.5e-2 < w_ref < 6e-2
    assert w <= max(w_ref * 1.5, 3.78e-2 * 1.5)


def test_fused_matches_reference_fused_kernel(cuda):
    A, B, bias = inputs(1024, 512, 512, init="lcg")
    theirs = ref_gemm(cuda, V_FUSED, A, B, bias)
    ours = run(cuda, A, B, bias, epilogue=b2g.EPI_BIAS_RELU)
    assert O.max_rel_diff(ours, theirs) <= 2 * 2.0 ** -11


def _epilogue_variants(acc, bias, alpha):
    """FP16 results of relu(alpha * acc + bias[n]) computed as one FMA (one rounding) and as a
    multiply then an add (two roundings, as src/gemm_bench.cu:380-383 is written)."""
    acc32 = acc.astype(np.float32)
    b32 = O.f16_to_f32(bias)[None, :]
    a32 = np.float32(alpha)
    # one rounding: the exact value alpha * acc + b (exact in FP64 here: acc has <= 10 bits,
    # alpha 24, b 11 within a few binades) rounded once to FP32
    fma = (acc32.astype(np.float64) * np.float64(a32) + b32.astype(np.float64)).astype(np.float32)
    muladd = (acc32 * a32).astype(np.float32) + b32
    return (O.f32_to_f16(np.maximum(fma, np.float32(0))),
            O.f32_to_f16(np.maximum(muladd, np.float32(0))))


def test_fused_epilogue_rounding_matches_reference_kernels(cuda):
    """Integer-valued inputs make every product and partial sum exact in FP32, so all kernels
    hold the same accumulator whatever their K order, and the fused epilogues can be compared
    bit for bit: ours, the reference's fused kernel (FUSE_EPILOGUE build) and its unfused
    bias_relu_kernel (on the exact plain product) must agree, and the test records which
    rounding (one FMA or multiply-then-add) the reference's compiled kernels perform."""
    torch = cuda
    M, N, K = 1024, 1024, 64
    rng = np.random.default_rng(5)
    A = O.f32_to_f16(rng.integers(-3, 4, (M, K)).astype(np.float32))
    B = O.f32_to_f16(rng.integers(-3, 4, (N, K)).astype(np.float32))
    bias = O.fill_uniform((N,), 7, 2, -4.0, 4.0)
    alpha = 0.1
    acc = np.rint(O.gemm_f64(A, B)).astype(np.int64)  # exact integer accumulators
    fma, muladd = _epilogue_variants(acc, bias, alpha)
    differ = int((fma != muladd).sum())
    assert differ > 0, "the inputs do not tell the two roundings apart"
    dA, dB, dbias = to_dev(torch, A), to_dev(torch, B), to_dev(torch, bias)
    dD = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    rc = O.ref().ref_gemm_launch(V_FUSED, dA.data_ptr(), dB.data_ptr(), dD.data_ptr(),
                                 dbias.data_ptr(), M, N, K, alpha, 2, 3, 3, 2,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    theirs_fused = to_host(dD)
    # the reference's unfused kernel on the exact plain product (exact in FP16: |acc| <= 576)
    dP = to_dev(torch, O.f32_to_f16(acc.astype(np.float32)))
    assert O.ref().ref_bias_relu(dP.data_ptr(), dbias.data_ptr(), M, N, alpha,
                                 torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    theirs_unfused = to_host(dP)
    kind = {True: "one FMA", False: "multiply then add"}
    for name, t in (("fused", theirs_fused), ("unfused", theirs_unfused)):
        is_fma, is_muladd = np.array_equal(t, fma), np.array_equal(t, muladd)
        print(f"reference {name} kernel: {kind[is_fma] if is_fma or is_muladd else 'neither'} "
              f"({differ} of {M * N} elements tell them apart)")
        assert is_fma or is_muladd
    ours = run(torch, A, B, bias, epilogue=b2g.EPI_BIAS_RELU, alpha=alpha)
    assert np.array_equal(ours, theirs_fused)
    dU = to_dev(torch, O.f32_to_f16(acc.astype(np.float32)))
    b2g.bias_relu(dU, dbias, alpha=alpha)
    b2g.sync_status()
    assert np.array_equal(to_host(dU), theirs_unfused)
