"""Helpers shared by the GPU tests: seeded inputs, launches through the C-ABI binding,
and comparisons against the CPU oracle."""
import numpy as np

import b2g
import oracle as O


def inputs(M, N, K, seed=0, lo=-1.0, hi=1.0, init="uniform"):
    """(A M x K, B N x K, bias N) as numpy uint16 FP16 bit patterns."""
    if init == "lcg":
        return O.fill_lcg(M, N, K)
    return (O.fill_uniform((M, K), seed, 0, lo, hi), O.fill_uniform((N, K), seed, 1, lo, hi),
            O.fill_uniform((N,), seed, 2, lo, hi))


def to_dev(torch, x, ld=None):
    """numpy uint16 (rows x cols) -> CUDA fp16 view with row pitch `ld` (>= cols)."""
    x = np.ascontiguousarray(x)
    t = torch.from_numpy(x.view(np.float16))
    if x.ndim == 1 or ld is None or ld == x.shape[1]:
        return t.cuda()
    rows, cols = x.shape
    buf = torch.zeros((rows, ld), dtype=torch.float16, device="cuda")
    buf[:, :cols].copy_(t.cuda())
    return buf[:, :cols]


def to_host(t):
    return np.ascontiguousarray(t.detach().cpu().numpy()).view(np.uint16)


def run(torch, A, B, bias=None, *, acc=b2g.ACC_F32, epilogue=b2g.EPI_NONE, alpha=1.0,
        tile=b2g.TILE_AUTO, stages=0, group=1, lda=None, ldb=None, ldd=None,
        b_layout=b2g.B_NK, splits=None):
    """Run the library GEMM on host inputs; returns D (numpy uint16, M x N)."""
    M, K = A.shape
    N = B.shape[0] if b_layout == b2g.B_NK else B.shape[1]
    dA = to_dev(torch, A, lda)
    dB = to_dev(torch, B, ldb)
    dbias = None if bias is None else to_dev(torch, bias)
    if ldd is None or ldd == N:
        dD = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    else:
        dD = torch.full((M, ldd), float("nan"), dtype=torch.float16, device="cuda")[:, :N]
    b2g.gemm(dA, dB, dD, dbias, b_layout=b_layout, acc=acc, epilogue=epilogue, alpha=alpha,
             tile=tile, stages=stages, group=group, splits=splits)
    b2g.sync_status()
    return to_host(dD)


def sample_rows(M, n):
    n = min(n, M)
    return sorted({int(r * M // n) for r in range(n)} | {M - 1})


def check_rows(A, B, D, rows, bias=None, alpha=1.0, epilogue=False, b_layout=0):
    """(relative Frobenius error, max |D-R|/max(1,|R|)) over the given rows vs FP64."""
    R = np.concatenate([O.gemm_f64(A, B, b_layout, r, r + 1) for r in rows])
    if epilogue:
        b = 0.0 if bias is None else O.f16_to_f32(bias)[None, :].astype(np.float64)
        R = np.maximum(R * alpha + b, 0.0)
    Dr = np.ascontiguousarray(D[rows])
    Df = O.f16_to_f32(Dr).astype(np.float64)
    assert np.all(np.isfinite(Df)), "non-finite output (unwritten or overflowed elements)"
    maxrel = float(np.max(np.abs(Df - R) / np.maximum(1.0, np.abs(R))))
    return O.frobenius_rel(Dr, R), maxrel
