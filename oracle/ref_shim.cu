// ref_shim.cu -- TEST INFRASTRUCTURE ONLY: the reference's own code, compiled from its
// unmodified source, behind a C-ABI so tests and the bench's reference arm can call it.
//
// The reference's single translation unit (src/gemm_bench.cu) is #included four times,
// each inside its own namespace with a different set of its compile-time switches
// (src/gemm_bench.cu:31-57, the four builds of scripts/build.ps1:48-62):
//     v_plain  : FUSE_EPILOGUE=0                     gemm_bench.exe
//     v_fused  : FUSE_EPILOGUE=1                     gemm_bench_fused.exe
//     v_f16acc : ACC_F16=1                           gemm_bench_f16acc.exe
//     v_k8     : MMA_K8=1                            gemm_bench_k8.exe (README best config)
// Its `main` is renamed so the file links as a library. Nothing of the reference is copied
// into this repository: the include path points at the read-only reference checkout and
// the output goes to oracle/_ref/ (git-ignored). Device code is compiled to compute_89
// PTX, so on a B200 the driver JIT-compiles the reference's sm_89 kernel unchanged.
//
// Exports (all return cudaError_t as int unless stated):
//   ref_spot_check     -> cpu_spot_check        src/gemm_bench.cu:672-696 (host FP64)
//   ref_float2half     -> host __float2half, the conversion the reference's init uses
//   ref_gemm_launch    -> gemm_kernel<...>      src/gemm_bench.cu:213-399, launched as run_cfg does
//   ref_max_rel_diff   -> max_rel_diff          src/gemm_bench.cu:648-664
//   ref_bias_relu      -> bias_relu_kernel      src/gemm_bench.cu:402-408
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <algorithm>
#include <chrono>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cublas_v2.h>

#ifndef REF_SRC
#error "REF_SRC must name the reference's src/gemm_bench.cu"
#endif

#define main ref_main_plain
namespace v_plain {
#define FUSE_EPILOGUE 0
#include REF_SRC
#undef FUSE_EPILOGUE
#undef ACC_F16
#undef MMA_K8
}  // namespace v_plain
#undef main

#define main ref_main_fused
namespace v_fused {
#define FUSE_EPILOGUE 1
#include REF_SRC
#undef FUSE_EPILOGUE
#undef ACC_F16
#undef MMA_K8
}  // namespace v_fused
#undef main

#define main ref_main_f16acc
namespace v_f16acc {
#define ACC_F16 1
#include REF_SRC
#undef FUSE_EPILOGUE
#undef ACC_F16
#undef MMA_K8
}  // namespace v_f16acc
#undef main

#define main ref_main_k8
namespace v_k8 {
#define MMA_K8 1
#include REF_SRC
#undef FUSE_EPILOGUE
#undef ACC_F16
#undef MMA_K8
}  // namespace v_k8
#undef main

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

// Launch one instantiation the way run_cfg does (src/gemm_bench.cu:462-488): opt-in smem
// attribute, grid (ceil(N/BN), ceil(M/BM)), block = warps*32, dynamic smem = SMEM_BYTES.
template <class Kern, class T>
int launch_one(Kern kern, int bm, int bn, const half* A, const half* B, half* D,
               const half* bias, int M, int N, int K, float alpha, int group,
               cudaStream_t s) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (T::SMEM_BYTES > optin) return (int)cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         T::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    dim3 grid((N + bn - 1) / bn, (M + bm - 1) / bm);
    kern<<<grid, T::THREADS, T::SMEM_BYTES, s>>>(A, B, D, bias, M, N, K, alpha, group);
    return (int)cudaGetLastError();
}

// The README's best configuration (README.md:439-440): tile 3 = 128x128x32 with 2x2 warps,
// 3 stages, swizzled smem; and the reference defaults tile 1 / 3 stages / pad layout.
#define REF_DISPATCH(NS)                                                                    \
    if (tile == 3 && stages == 3 && layout == 2) {                                          \
        using T = NS::Traits<128, 128, 32, 2, 2, 3, NS::LAYOUT_SWZ>;                        \
        return launch_one<decltype(&NS::gemm_kernel<128, 128, 32, 2, 2, 3, NS::LAYOUT_SWZ>), \
                          T>(&NS::gemm_kernel<128, 128, 32, 2, 2, 3, NS::LAYOUT_SWZ>, 128,   \
                             128, a, b, d, bias, M, N, K, alpha, group, s);                  \
    }                                                                                       \
    if (tile == 1 && stages == 3 && layout == 1) {                                          \
        using T = NS::Traits<128, 128, 32, 2, 4, 3, NS::LAYOUT_PAD>;                        \
        return launch_one<decltype(&NS::gemm_kernel<128, 128, 32, 2, 4, 3, NS::LAYOUT_PAD>), \
                          T>(&NS::gemm_kernel<128, 128, 32, 2, 4, 3, NS::LAYOUT_PAD>, 128,   \
                             128, a, b, d, bias, M, N, K, alpha, group, s);                  \
    }                                                                                       \
    return (int)cudaErrorInvalidValue;

}  // namespace

// variant: 0 plain, 1 fused (alpha*acc + bias, ReLU), 2 FP16 accumulate, 3 MMA_K8.
// The reference kernel needs K % 32 == 0 (src/gemm_bench.cu:746) and 16-byte aligned rows;
// its half2 epilogue store also needs N even. Those are checked here and rejected with
// cudaErrorInvalidValue instead of launching.
REF_API int ref_gemm_launch(int variant, const void* A, const void* B, void* D,
                            const void* bias, int M, int N, int K, float alpha, int group,
                            int tile, int stages, int layout, void* stream) {
    if (M <= 0 || N <= 0 || K <= 0 || K % 32 != 0 || N % 2 != 0) return (int)cudaErrorInvalidValue;
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)D) & 15) return (int)cudaErrorInvalidValue;
    const half* a = (const half*)A;
    const half* b = (const half*)B;
    half* d = (half*)D;
    const half* bias_h = (const half*)bias;
    (void)bias_h;
    cudaStream_t s = (cudaStream_t)stream;
    switch (variant) {
        case 0: { const half* bias = bias_h; REF_DISPATCH(v_plain) }
        case 1: { const half* bias = bias_h; REF_DISPATCH(v_fused) }
        case 2: { const half* bias = bias_h; REF_DISPATCH(v_f16acc) }
        case 3: { const half* bias = bias_h; REF_DISPATCH(v_k8) }
    }
    return (int)cudaErrorInvalidValue;
}

REF_API int ref_max_rel_diff(const void* x, const void* y, size_t n, float* out_dev,
                             void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(out_dev, 0, sizeof(float), s);
    if (e != cudaSuccess) return (int)e;
    v_plain::max_rel_diff<<<256, 256, 0, s>>>((const half*)x, (const half*)y, n, out_dev);
    return (int)cudaGetLastError();
}

REF_API int ref_bias_relu(void* D, const void* bias, int M, int N, float alpha, void* stream) {
    const size_t nD = (size_t)M * N;
    constexpr int t = 256;
    v_plain::bias_relu_kernel<<<(unsigned)((nD + t - 1) / t), t, 0, (cudaStream_t)stream>>>(
        (half*)D, (const half*)bias, M, N, alpha);
    return (int)cudaGetLastError();
}

// Host-only: the reference's FP64 spot check on caller-owned FP16 arrays (B is N x K).
REF_API double ref_spot_check(const uint16_t* A, const uint16_t* B, const uint16_t* D,
                              const uint16_t* bias, int M, int N, int K, int samples,
                              int fused, float alpha, int* worst_m, int* worst_n) {
    std::vector<half> hA((size_t)M * K), hB((size_t)N * K), hD((size_t)M * N), hBias(N);
    std::memcpy(hA.data(), A, hA.size() * 2);
    std::memcpy(hB.data(), B, hB.size() * 2);
    std::memcpy(hD.data(), D, hD.size() * 2);
    if (bias) std::memcpy(hBias.data(), bias, hBias.size() * 2);
    return v_plain::cpu_spot_check(hA, hB, hD, hBias, M, N, K, samples, fused != 0, alpha,
                                   worst_m, worst_n);
}

// Host-only: the reference's float -> half conversion (cuda_fp16.h host path).
REF_API uint16_t ref_float2half(float f) {
    half h = __float2half(f);
    uint16_t u;
    std::memcpy(&u, &h, 2);
    return u;
}

// Host-only, multi-threaded timing harness for the reference arm of bench.py: runs the
// reference's cpu_spot_check -- the only CPU implementation of D = A*B in the reference --
// over `rows` full output rows starting at row m0 (every element of those rows, FP64),
// split across `threads` host threads. Each thread gets its own row panel of A so the
// reference function sees a dense (rows_t x N x K) problem. Returns elapsed seconds.
REF_API double ref_cpu_rows(const uint16_t* A, const uint16_t* B, const uint16_t* D, int M,
                            int N, int K, int m0, int rows, int threads);

#include <thread>

REF_API double ref_cpu_rows(const uint16_t* A, const uint16_t* B, const uint16_t* D, int M,
                            int N, int K, int m0, int rows, int threads) {
    if (threads < 1) threads = 1;
    if (rows > M - m0) rows = M - m0;
    if (threads > rows) threads = rows > 0 ? rows : 1;
    std::vector<half> hB((size_t)N * K), hBias(N);
    std::memcpy(hB.data(), B, hB.size() * 2);
    struct Panel { std::vector<half> a, d; int r0, nr; double worst; int wm, wn; };
    std::vector<Panel> panels(threads);
    for (int t = 0; t < threads; ++t) {
        Panel& p = panels[t];
        p.r0 = m0 + (int)((long long)rows * t / threads);
        p.nr = m0 + (int)((long long)rows * (t + 1) / threads) - p.r0;
        p.a.resize((size_t)p.nr * K);
        p.d.resize((size_t)p.nr * N);
        std::memcpy(p.a.data(), A + (size_t)p.r0 * K, p.a.size() * 2);
        std::memcpy(p.d.data(), D + (size_t)p.r0 * N, p.d.size() * 2);
    }
    auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&, t] {
            Panel& p = panels[t];
            p.worst = v_plain::cpu_spot_check(p.a, hB, p.d, hBias, p.nr, N, K, p.nr * N,
                                              false, 1.0f, &p.wm, &p.wn);
        });
    for (auto& th : pool) th.join();
    auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}
