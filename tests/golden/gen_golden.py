"""Generate the golden fixtures of tests/golden/ from the reference's OWN code.

Run in a container that has the reference checkout (it needs oracle/_ref/libref.so, which
oracle/Makefile compiles from the reference's unmodified src/gemm_bench.cu):

    make -C oracle && python tests/golden/gen_golden.py

Outputs (committed):
  float2half.json  -- host __float2half results (the conversion the reference's init uses)
                      for edge-case and random floats: [[f32_bits, f16_bits], ...]
  spot_check.json  -- the reference's cpu_spot_check (src/gemm_bench.cu:672-696) on FP16
                      inputs from the reference's LCG init (src/gemm_bench.cu:760-765) and
                      from the seeded uniform generator, with D = FP16(FP64 product) plus
                      planted bit flips, fused and plain; each case stores the reference's
                      (worst, worst_m, worst_n).
The tests regenerate the same inputs with the CPU oracle and require the oracle's restated
spot check to reproduce the reference's answers exactly.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

CASES = [
    # M, N, K, init, samples, fused, alpha, plants [(m, n, xor_bits)]
    (64, 64, 32, "lcg", 512, 0, 1.0, []),
    (64, 64, 32, "lcg", 512, 0, 1.0, [(3, 5, 0x0200)]),
    (96, 80, 64, "lcg", 7, 0, 1.0, [(0, 0, 0x0100)]),
    (96, 80, 64, "lcg", 7680, 1, 1.0, [(10, 11, 0x0400)]),
    (128, 96, 128, "uniform:0:-1:1", 1000, 0, 1.0, [(127, 95, 0x0001)]),
    (128, 96, 128, "uniform:2:-0.5:0.5", 333, 1, 0.5, []),
    (33, 17, 96, "uniform:5:-1:1", 561, 1, 2.0, [(32, 16, 0x8000)]),
    (1, 1, 32, "lcg", 1, 0, 1.0, []),
    (200, 300, 256, "uniform:1:-1:1", 4096, 0, 1.0, [(199, 299, 0x0040), (0, 1, 0x0010)]),
]


def make_inputs(M, N, K, init):
    if init == "lcg":
        return O.fill_lcg(M, N, K)
    _, seed, lo, hi = init.split(":")
    seed, lo, hi = int(seed), float(lo), float(hi)
    A = O.fill_uniform((M, K), seed, 0, lo, hi)
    B = O.fill_uniform((N, K), seed, 1, lo, hi)
    bias = O.fill_uniform((N,), seed, 2, lo, hi)
    return A, B, bias


def make_D(A, B, bias, fused, alpha, plants):
    R = O.gemm_f64(A, B)
    if fused:
        R = np.maximum(R * alpha + O.f16_to_f32(bias)[None, :].astype(np.float64), 0.0)
    D = O.f32_to_f16(R.astype(np.float32))
    for m, n, x in plants:
        D[m, n] ^= x
    return D


def main():
    assert O.ref_available(), "oracle/_ref/libref.so missing: run make -C oracle"
    R = O.ref()
    rng = np.random.default_rng(1234)
    floats = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 0.5, 65504.0, 65519.996, 65520.0, 1e6, -1e6,
                  5.96e-8, 2.98e-8, 2.99e-8, 6.1e-5, 6.0e-5, np.inf, -np.inf], np.float32),
        (rng.standard_normal(400) * 10.0 ** rng.integers(-9, 6, 400)).astype(np.float32),
        ((np.arange(1024) / np.float32(1023.0)) - np.float32(0.5)).astype(np.float32),
    ]).astype(np.float32)
    f2h = [[int(f.view(np.uint32)), int(R.ref_float2half(float(f)))] for f in floats]
    with open(os.path.join(HERE, "float2half.json"), "w") as fh:
        json.dump(f2h, fh)

    out = []
    for M, N, K, init, samples, fused, alpha, plants in CASES:
        A, B, bias = make_inputs(M, N, K, init)
        D = make_D(A, B, bias, fused, alpha, plants)
        w, wm, wn = O.ref_spot_check(A, B, D, bias, samples, bool(fused), alpha)
        out.append(dict(M=M, N=N, K=K, init=init, samples=samples, fused=fused, alpha=alpha,
                        plants=plants, worst=w, worst_m=wm, worst_n=wn))
    with open(os.path.join(HERE, "spot_check.json"), "w") as fh:
        json.dump(out, fh, indent=1)
    print(f"wrote {len(f2h)} float2half and {len(out)} spot_check cases")


if __name__ == "__main__":
    main()
