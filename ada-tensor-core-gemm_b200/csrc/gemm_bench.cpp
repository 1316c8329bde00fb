// gemm_bench.cpp -- command-line driver of the B200 GEMM, with the reference CLI's flags.
//
// Mirrors the reference's gemm_bench (src/gemm_bench.cu:698-868): same flags, same
// defaults where they still mean something, same fail-fast behaviour (unknown flag ->
// exit 2), the same whitespace-separated result table (column order is the contract that
// scripts/sweep.ps1:33-51 parses; new columns are appended at the end), the same `SOAK,`
// CSV lines, a cuBLAS comparison column, the device max-rel check (--check) and the FP64
// host spot check (--cpu S). All GPU work goes through the library's C-ABI (b2g.h).
//
// Differences, all because the hardware path changed:
//   --tile    selects B200 tiles: -1 = from the shape (default), 0 = 128x128, 1 = 128x256,
//             2 = 256x256 2-SM pair, 3 = 128x64, 4 = 256x512 2-SM pair, 5 = swap-AB,
//             6 = 256x128 2-SM pair
//   --layout  only 2 (swizzle) exists on sm_100a: TMA writes the 128-byte-swizzled layout
//             tcgen05.mma reads; 0 / 1 print a SKIP row like an unsupported config
//   --stages  shared-memory ring depth 2..8 (0 = deepest that fits); --sweep runs 2..8
//   no K % 32 restriction (TMA zero-fills the K tail); A/B leading dimensions are padded
//             to a multiple of 8 elements when K is not (16-byte TMA row strides)
// New flags: --acc f32|f16, --fused, --b-layout nk|kn, --init ref|uniform, --seed S,
//            --dist LO,HI, --frob ROWS, --json, --splits S, --gpus N, --allgather.
//   --gpus N  one GEMM split by M-row panels over devices 0..N-1 (b2g_gemm_multi: A and D
//             by rows, B copied to every device); --allgather then copies every panel to
//             every device over NVLink (b2g_allgather_rows), timed on its own, and then
//             times the GEMM with the all-gather fused into its epilogue
//             (b2g_gemm_multi_allgather).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "b2g.h"

#define CUDA_CHECK(x)                                                                   \
    do {                                                                                \
        cudaError_t e_ = (x);                                                           \
        if (e_ != cudaSuccess) {                                                        \
            fprintf(stderr, "CUDA error %s:%d: %s\n", __FILE__, __LINE__,               \
                    cudaGetErrorString(e_));                                            \
            exit(1);                                                                    \
        }                                                                               \
    } while (0)

namespace {

struct Args {
    int M = 4096, N = 4096, K = 4096;
    int tile = -1, stages = 0, layout = 2, group = 0;  // -1 / 0 = chosen from the shape
    int iters = 50, warmup = 20;
    int splits = -1;    // split-K factor: -1 = b2g_gemm (automatic), else b2g_gemm_splitk
    int gpus = 1;       // devices for the M-panel multi-GPU run (b2g_gemm_multi)
    bool allgather = false;
    int cpu = 0;        // output elements verified by the FP64 host spot check
    int frob = 0;       // rows of D checked by an FP64 relative Frobenius norm
    double soak = 0;    // seconds of back-to-back launches (0 = fixed iters)
    double window = 2.0;
    bool check = false, ref = true, sweep = false, unfused = false, gsweep = false;
    bool fused = false, json = false;
    int acc = B2G_ACC_F32, b_layout = B2G_B_NK;
    bool init_ref = true;
    unsigned long long seed = 0;
    double lo = -0.5, hi = 0.5;
};

float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, x;
    if (e == 0x1F) {
        x = sign | 0x7F800000u | (m << 13);
    } else if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            int s = 0;
            while (!(m & 0x400u)) { m <<= 1; ++s; }
            x = sign | ((uint32_t)(113 - s) << 23) | ((m & 0x3FFu) << 13);
        }
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

// FP64 spot check with the reference's semantics (src/gemm_bench.cu:666-696): `samples`
// output elements at a fixed odd stride, FP64 dot products of the FP16 inputs, relative
// error |got - ref| / max(1, |ref|), bias + ReLU applied when an epilogue ran.
double spot_check(const std::vector<uint16_t>& A, long long lda, const std::vector<uint16_t>& B,
                  long long ldb, int b_layout, const std::vector<uint16_t>& D, long long ldd,
                  const std::vector<uint16_t>& bias, int M, int N, int K, int samples, bool epi,
                  float alpha, int* wm, int* wn) {
    double worst = 0.0;
    *wm = *wn = -1;
    const long long total = (long long)M * N;
    const long long stride = (total / std::max(1, samples)) | 1;
    long long idx = 0;
    for (long long s = 0; s < samples && s < total; ++s, idx = (idx + stride) % total) {
        const int m = (int)(idx / N), n = (int)(idx % N);
        double acc = 0.0;
        for (int k = 0; k < K; ++k) {
            const uint16_t b = b_layout == B2G_B_NK ? B[(size_t)n * ldb + k] : B[(size_t)k * ldb + n];
            acc += (double)h2f(A[(size_t)m * lda + k]) * (double)h2f(b);
        }
        if (epi) {
            acc = acc * alpha + (double)h2f(bias[n]);
            if (acc < 0) acc = 0;
        }
        const double got = (double)h2f(D[(size_t)m * ldd + n]);
        const double rel = fabs(got - acc) / std::max(1.0, fabs(acc));
        if (rel > worst) { worst = rel; *wm = m; *wn = n; }
    }
    return worst;
}

// Relative Frobenius error over `rows` rows spread evenly through D (FP64 reference).
double frobenius_rows(const std::vector<uint16_t>& A, long long lda, const std::vector<uint16_t>& B,
                      long long ldb, int b_layout, const std::vector<uint16_t>& D, long long ldd,
                      const std::vector<uint16_t>& bias, int M, int N, int K, int rows, bool epi,
                      float alpha) {
    double num = 0, den = 0;
    rows = std::min(rows, M);
    std::vector<double> bcol((size_t)K);
    std::vector<double> ref((size_t)N);
    for (int r = 0; r < rows; ++r) {
        const int m = (int)((long long)r * M / rows);
        for (int n = 0; n < N; ++n) {
            double acc = 0;
            for (int k = 0; k < K; ++k) {
                const uint16_t b = b_layout == B2G_B_NK ? B[(size_t)n * ldb + k] : B[(size_t)k * ldb + n];
                acc += (double)h2f(A[(size_t)m * lda + k]) * (double)h2f(b);
            }
            if (epi) acc = std::max(0.0, acc * alpha + (double)h2f(bias[n]));
            const double d = (double)h2f(D[(size_t)m * ldd + n]) - acc;
            num += d * d;
            den += acc * acc;
        }
    }
    return den > 0 ? sqrt(num / den) : sqrt(num);
}

const char* tile_name(int t) {
    return t == 0 ? "128x128x64" : t == 1 ? "128x256x64" : t == 2 ? "256x256x64"
         : t == 3 ? "128x64x64" : t == 4 ? "256x512x64" : t == 5 ? "swapAB"
         : t == 6 ? "256x128x64" : "auto";
}

void usage(const char* argv0) {
    printf("usage: %s [--m M --n N --k K] [--tile 0..6] [--stages 0|2..8]\n"
           "       [--layout 2] [--group G] [--iters N] [--warmup N] [--check] [--cpu S]\n"
           "       [--noref] [--sweep] [--gsweep] [--unfused] [--soak SEC] [--window SEC]\n"
           "       [--acc f32|f16] [--fused] [--b-layout nk|kn] [--init ref|uniform]\n"
           "       [--seed S] [--dist LO,HI] [--frob ROWS] [--json] [--splits S]\n"
           "       [--gpus N [--allgather]]\n"
           "  --check    compare against cuBLAS on the device (max |x-y|/max(1,|y|))\n"
           "  --cpu S    verify S output elements against an FP64 host dot product\n"
           "  --frob R   FP64 relative Frobenius error over R rows spread through D\n"
           "  tile -1 = chosen from the shape (default)\n"
           "       0 = 128x128x64  1 CTA, UMMA 128x128, TMEM 2x128 cols\n"
           "       1 = 128x256x64  1 CTA, UMMA 128x256, TMEM 2x256 cols\n"
           "       2 = 256x256x64  2-CTA pair (cta_group::2), UMMA 256x256\n"
           "       3 = 128x64x64   1 CTA, UMMA 128x64, TMEM 2x64 cols\n"
           "       4 = 256x512x64  2-CTA pair, two UMMA 256x256 halves, TMEM 512 cols\n"
           "       5 = swapAB      small M: UMMA 128 x MT (MT = 16..64 rows of A), B rows on M\n"
           "                       (narrow form, ~N/SMs rows of B per CTA, when N is small)\n"
           "       6 = 256x128x64  2-CTA pair, UMMA 256x128\n"
           "  --splits S split-K factor (0 automatic, 1 none, S >= 2 forced; default: automatic)\n"
           "  --gpus N   M-row panels over devices 0..N-1 (b2g_gemm_multi), B on every device;\n"
           "             --allgather then gathers D on every device over NVLink (timed apart)\n"
           "             and times the GEMM with the gather fused into its epilogue\n"
           "  --stages   shared-memory ring depth (0 = deepest that fits)\n"
           "  --group G  L2 rasterization: G M-tiles walked column-major (1 = row-major)\n"
           "  --sweep    stages 2..8 at fixed tile/group;  --gsweep  group 1,2,4,8,16\n"
           "  --acc      f32 (default) or f16 accumulation; --fused alpha*acc+bias+ReLU\n"
           "  --init     ref = the reference's LCG (default), uniform = seeded U[LO,HI]\n",
           argv0);
}

// --gpus N: the M-panel plan over devices 0..N-1 through b2g_gemm_multi (and, with
// --allgather, b2g_allgather_rows). Device time per step is the maximum over the devices of
// CUDA-event time on each device's stream, as the multi-GPU timing rule asks.
int run_multi(const Args& a, const std::vector<uint16_t>& hA, const std::vector<uint16_t>& hB,
              const std::vector<uint16_t>& hBias, long long lda, long long ldb, long long ldd) {
    int ndev = 0;
    CUDA_CHECK(cudaGetDeviceCount(&ndev));
    if (a.gpus < 1 || a.gpus > ndev) {
        fprintf(stderr, "--gpus %d: %d device(s) visible\n", a.gpus, ndev);
        return 2;
    }
    if (a.soak > 0 || a.sweep || a.gsweep || a.unfused || a.splits >= 0) {
        fprintf(stderr, "--gpus runs one configuration: no --soak/--sweep/--gsweep/--unfused/--splits\n");
        return 2;
    }
    const int G = a.gpus;
    const size_t brows = a.b_layout == B2G_B_NK ? (size_t)a.N : (size_t)a.K;
    const size_t nB = brows * (size_t)ldb, nFull = (size_t)a.M * (size_t)ldd;
    std::vector<int> devs(G);
    std::vector<void*> dA(G), dB(G), dD(G), dBias(G), dFull(G, nullptr);
    std::vector<void*> streams(G);
    std::vector<cudaEvent_t> t0(G), t1(G);
    for (int g = 0; g < G; ++g) {
        devs[g] = g;
        const int r0 = (int)((long long)a.M * g / G), r1 = (int)((long long)a.M * (g + 1) / G);
        const size_t rows = (size_t)(r1 - r0);
        CUDA_CHECK(cudaSetDevice(g));
        CUDA_CHECK(cudaMalloc(&dA[g], std::max<size_t>(rows * lda, 8) * 2));
        CUDA_CHECK(cudaMalloc(&dB[g], std::max<size_t>(nB, 8) * 2));
        CUDA_CHECK(cudaMalloc(&dD[g], std::max<size_t>(rows * ldd, 8) * 2));
        CUDA_CHECK(cudaMalloc(&dBias[g], hBias.size() * 2));
        if (a.allgather) CUDA_CHECK(cudaMalloc(&dFull[g], std::max<size_t>(nFull, 8) * 2));
        if (rows) CUDA_CHECK(cudaMemcpy(dA[g], &hA[(size_t)r0 * lda], rows * lda * 2,
                                        cudaMemcpyHostToDevice));
        CUDA_CHECK(cudaMemcpy(dB[g], hB.data(), nB * 2, cudaMemcpyHostToDevice));
        CUDA_CHECK(cudaMemcpy(dBias[g], hBias.data(), hBias.size() * 2, cudaMemcpyHostToDevice));
        cudaStream_t s;
        CUDA_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        streams[g] = s;
        CUDA_CHECK(cudaEventCreate(&t0[g]));
        CUDA_CHECK(cudaEventCreate(&t1[g]));
    }
    const int epi = a.fused ? B2G_EPI_BIAS_RELU : B2G_EPI_NONE;
    auto launch = [&](int sync) {
        return b2g_gemm_multi(G, devs.data(), (const void* const*)dA.data(),
                              (const void* const*)dB.data(), dD.data(),
                              a.fused ? (const void* const*)dBias.data() : nullptr, a.M, a.N, a.K,
                              lda, ldb, ldd, a.b_layout, a.acc, epi, 1.0f, a.tile, a.stages,
                              a.group, streams.data(), sync);
    };
    auto sync_all = [&]() {
        for (int g = 0; g < G; ++g) {
            CUDA_CHECK(cudaSetDevice(g));
            CUDA_CHECK(cudaStreamSynchronize((cudaStream_t)streams[g]));
        }
    };
    // time `body` over `n` repetitions: events on every device's stream, max over devices
    auto timed = [&](int n, auto&& body) -> double {
        sync_all();
        for (int g = 0; g < G; ++g) {
            CUDA_CHECK(cudaSetDevice(g));
            CUDA_CHECK(cudaEventRecord(t0[g], (cudaStream_t)streams[g]));
        }
        for (int i = 0; i < n; ++i)
            if (body() != B2G_OK) {
                fprintf(stderr, "error: %s\n", b2g_last_error());
                exit(1);
            }
        double worst = 0;
        for (int g = 0; g < G; ++g) {
            CUDA_CHECK(cudaSetDevice(g));
            CUDA_CHECK(cudaEventRecord(t1[g], (cudaStream_t)streams[g]));
        }
        for (int g = 0; g < G; ++g) {
            CUDA_CHECK(cudaSetDevice(g));
            CUDA_CHECK(cudaEventSynchronize(t1[g]));
            float ms = 0;
            CUDA_CHECK(cudaEventElapsedTime(&ms, t0[g], t1[g]));
            worst = std::max(worst, (double)ms);
        }
        return worst / std::max(1, n);
    };
    for (int i = 0; i < a.warmup; ++i)
        if (launch(0) != B2G_OK) {
            fprintf(stderr, "error: %s\n", b2g_last_error());
            return 1;
        }
    if (launch(1) != B2G_OK) {  // one checked launch: every device's status word
        fprintf(stderr, "error: %s\n", b2g_last_error());
        return 1;
    }
    const double flop = 2.0 * a.M * a.N * a.K;
    const double ms = timed(a.iters, [&]() { return launch(0); });
    const double tflops = flop / (ms * 1e-3) / 1e12;
    if (launch(1) != B2G_OK) {
        fprintf(stderr, "error: %s\n", b2g_last_error());
        return 1;
    }
    double ag_ms = -1, ag_gbs = -1;
    if (a.allgather) {
        auto gather = [&]() {
            return b2g_allgather_rows(G, devs.data(), dD.data(), dFull.data(), a.M, a.N, ldd,
                                      streams.data(), 0);
        };
        for (int i = 0; i < std::max(1, a.warmup / 4); ++i)
            if (gather() != B2G_OK) {
                fprintf(stderr, "error: %s\n", b2g_last_error());
                return 1;
            }
        ag_ms = timed(std::max(1, a.iters / 4), gather);
        // bytes each device receives from its peers per gather
        const double recv = (double)a.M * a.N * 2.0 * (G - 1) / G;
        ag_gbs = recv / (ag_ms * 1e-3) / 1e9;
    }
    sync_all();

    // assemble D from the panels; with --allgather, every device's gathered copy must equal it
    std::vector<uint16_t> hD(nFull);
    for (int g = 0; g < G; ++g) {
        const int r0 = (int)((long long)a.M * g / G), r1 = (int)((long long)a.M * (g + 1) / G);
        CUDA_CHECK(cudaSetDevice(g));
        if (r1 > r0)
            CUDA_CHECK(cudaMemcpy(&hD[(size_t)r0 * ldd], dD[g], (size_t)(r1 - r0) * ldd * 2,
                                  cudaMemcpyDeviceToHost));
    }
    // every device's D_full must equal the assembled panels: whole copies up to 256 MiB,
    // else 257 rows spread through D
    auto full_matches = [&]() -> int {
        const bool whole = nFull * 2 <= (256u << 20);
        std::vector<uint16_t> row((size_t)ldd);
        for (int g = 0; g < G; ++g) {
            CUDA_CHECK(cudaSetDevice(g));
            if (whole) {
                std::vector<uint16_t> hF(nFull);
                CUDA_CHECK(cudaMemcpy(hF.data(), dFull[g], nFull * 2, cudaMemcpyDeviceToHost));
                if (memcmp(hF.data(), hD.data(), nFull * 2) != 0) return 0;
            } else {
                for (int r = 0; r <= 256; ++r) {
                    const size_t m = (size_t)((long long)r * (a.M - 1) / 256);
                    CUDA_CHECK(cudaMemcpy(row.data(), (const uint16_t*)dFull[g] + m * ldd,
                                          (size_t)ldd * 2, cudaMemcpyDeviceToHost));
                    if (memcmp(row.data(), &hD[m * ldd], (size_t)a.N * 2) != 0) return 0;
                }
            }
        }
        return 1;
    };
    int gather_ok = -1, fused_ok = -1;
    double fz_ms = -1, fz_tflops = -1;
    if (a.allgather) {
        gather_ok = full_matches();
        // the same GEMM with the all-gather fused into the epilogue (b2g_gemm_multi_allgather)
        if (a.N % 8 == 0 && ldd % 8 == 0) {
            for (int g = 0; g < G; ++g) {  // clear the copies the separate gather wrote
                CUDA_CHECK(cudaSetDevice(g));
                CUDA_CHECK(cudaMemset(dFull[g], 0xFF, std::max<size_t>(nFull, 8) * 2));
            }
            sync_all();
            auto fused = [&]() {
                return b2g_gemm_multi_allgather(
                    G, devs.data(), (const void* const*)dA.data(), (const void* const*)dB.data(),
                    dFull.data(), a.fused ? (const void* const*)dBias.data() : nullptr, a.M, a.N,
                    a.K, lda, ldb, ldd, a.b_layout, a.acc, epi, 1.0f, a.tile, a.stages, a.group,
                    streams.data(), 0);
            };
            for (int i = 0; i < a.warmup; ++i)
                if (fused() != B2G_OK) {
                    fprintf(stderr, "error: %s\n", b2g_last_error());
                    return 1;
                }
            fz_ms = timed(a.iters, fused);
            fz_tflops = flop / (fz_ms * 1e-3) / 1e12;
            sync_all();
            for (int g = 0; g < G; ++g) {
                CUDA_CHECK(cudaSetDevice(g));
                if (b2g_sync_status(streams[g]) != B2G_OK) {
                    fprintf(stderr, "error: %s\n", b2g_last_error());
                    return 1;
                }
            }
            fused_ok = full_matches();
        }
    }
    const bool epi_on = a.fused;
    double cpurel = -1, frob = -1;
    int wm = -1, wn = -1;
    if (a.cpu > 0)
        cpurel = spot_check(hA, lda, hB, ldb, a.b_layout, hD, ldd, hBias, a.M, a.N, a.K, a.cpu,
                            epi_on, 1.0f, &wm, &wn);
    if (a.frob > 0)
        frob = frobenius_rows(hA, lda, hB, ldb, a.b_layout, hD, ldd, hBias, a.M, a.N, a.K,
                              a.frob, epi_on, 1.0f);

    printf("# problem       : M=%d N=%d K=%d over %d GPU(s), M-row panels, B on every device\n",
           a.M, a.N, a.K, G);
    printf("gpus=%d  tile=%d  ms=%.4f  TFLOP/s=%.2f  per_gpu=%.2f", G, a.tile, ms, tflops,
           tflops / G);
    if (ag_ms >= 0)
        printf("  allgather_ms=%.4f  allgather_GB/s=%.1f  gather=%s", ag_ms, ag_gbs,
               gather_ok ? "OK" : "FAIL");
    if (fz_ms >= 0)
        printf("  fused_ms=%.4f  fused_TFLOP/s=%.2f  fused=%s", fz_ms, fz_tflops,
               fused_ok ? "OK" : "FAIL");
    if (cpurel >= 0)
        printf("  cpu=%.2e%s(worst m=%d n=%d)", cpurel, cpurel < 3e-2 ? " OK " : " FAIL ", wm, wn);
    if (frob >= 0) printf("  frob=%.2e", frob);
    printf("\n");
    if (a.json)
        printf("{\"M\": %d, \"N\": %d, \"K\": %d, \"gpus\": %d, \"tile\": %d, \"acc\": \"%s\", "
               "\"ms\": %.5f, \"tflops\": %.3f, \"tflops_per_gpu\": %.3f, \"allgather_ms\": %.5f, "
               "\"allgather_gbs\": %.2f, \"gather_ok\": %d, \"fused_ms\": %.5f, "
               "\"fused_tflops\": %.3f, \"fused_ok\": %d, \"cpu_maxrel\": %.3e, "
               "\"frob_rel\": %.3e}\n",
               a.M, a.N, a.K, G, a.tile, a.acc == B2G_ACC_F32 ? "f32" : "f16", ms, tflops,
               tflops / G, ag_ms, ag_gbs, gather_ok, fz_ms, fz_tflops, fused_ok, cpurel, frob);
    fflush(stdout);
    for (int g = 0; g < G; ++g) {
        cudaSetDevice(g);
        cudaFree(dA[g]); cudaFree(dB[g]); cudaFree(dD[g]); cudaFree(dBias[g]);
        if (dFull[g]) cudaFree(dFull[g]);
        cudaStreamDestroy((cudaStream_t)streams[g]);
        cudaEventDestroy(t0[g]);
        cudaEventDestroy(t1[g]);
    }
    return (gather_ok == 0 || fused_ok == 0 || (cpurel >= 3e-2) || (frob >= 0 && frob > 1e-2))
               ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        auto eq = [&](const char* s) { return strcmp(argv[i], s) == 0; };
        auto sval = [&]() -> const char* { return (i + 1 < argc) ? argv[++i] : ""; };
        auto val = [&]() -> int { return atoi(sval()); };
        auto dval = [&]() -> double { return atof(sval()); };
        if (eq("--m")) a.M = val();
        else if (eq("--n")) a.N = val();
        else if (eq("--k")) a.K = val();
        else if (eq("--tile")) a.tile = val();
        else if (eq("--stages")) a.stages = val();
        else if (eq("--layout")) a.layout = val();
        else if (eq("--iters")) a.iters = val();
        else if (eq("--warmup")) a.warmup = val();
        else if (eq("--group")) a.group = val();
        else if (eq("--splits")) a.splits = val();
        else if (eq("--gpus")) a.gpus = val();
        else if (eq("--allgather")) a.allgather = true;
        else if (eq("--cpu")) a.cpu = val();
        else if (eq("--frob")) a.frob = val();
        else if (eq("--soak")) a.soak = dval();
        else if (eq("--window")) a.window = dval();
        else if (eq("--check")) a.check = true;
        else if (eq("--noref")) a.ref = false;
        else if (eq("--sweep")) a.sweep = true;
        else if (eq("--gsweep")) a.gsweep = true;
        else if (eq("--unfused")) a.unfused = true;
        else if (eq("--fused")) a.fused = true;
        else if (eq("--json")) a.json = true;
        else if (eq("--acc")) {
            std::string v = sval();
            if (v == "f32") a.acc = B2G_ACC_F32;
            else if (v == "f16") a.acc = B2G_ACC_F16;
            else { fprintf(stderr, "--acc must be f32 or f16\n"); return 2; }
        } else if (eq("--b-layout")) {
            std::string v = sval();
            if (v == "nk") a.b_layout = B2G_B_NK;
            else if (v == "kn") a.b_layout = B2G_B_KN;
            else { fprintf(stderr, "--b-layout must be nk or kn\n"); return 2; }
        } else if (eq("--init")) {
            std::string v = sval();
            if (v == "ref") a.init_ref = true;
            else if (v == "uniform") a.init_ref = false;
            else { fprintf(stderr, "--init must be ref or uniform\n"); return 2; }
        } else if (eq("--seed")) a.seed = strtoull(sval(), nullptr, 10);
        else if (eq("--dist")) {
            if (sscanf(sval(), "%lf,%lf", &a.lo, &a.hi) != 2) {
                fprintf(stderr, "--dist needs LO,HI\n");
                return 2;
            }
        } else if (eq("--help")) {
            usage(argv[0]);
            return 0;
        } else {
            // a typo'd flag must stop the run: otherwise a long measurement runs with defaults
            fprintf(stderr, "unknown option '%s' (try --help)\n", argv[i]);
            return 2;
        }
    }
    if (a.M < 0 || a.N < 0 || a.K < 0) { fprintf(stderr, "M, N, K must be >= 0\n"); return 1; }

    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    cudaDeviceProp prop{};
    CUDA_CHECK(cudaGetDeviceProperties(&prop, dev));

    // leading dimensions: TMA wants 16-byte row strides for A and B
    const long long lda = ((long long)a.K + 7) / 8 * 8;
    const long long ldb = a.b_layout == B2G_B_NK ? lda : ((long long)a.N + 7) / 8 * 8;
    const long long ldd = a.N;
    const long long brows = a.b_layout == B2G_B_NK ? a.N : a.K;
    const size_t nA = (size_t)a.M * lda, nB = (size_t)brows * ldb, nD = (size_t)a.M * ldd;
    std::vector<uint16_t> hA(nA, 0), hB(nB, 0), hBias((size_t)std::max(a.N, 1), 0);
    {
        // logical (unpadded) data first, then spread into the padded rows
        std::vector<uint16_t> tA((size_t)a.M * a.K), tB((size_t)a.N * a.K);
        if (a.init_ref) {
            b2g_fill_lcg_f16(tA.data(), (long long)tA.size(), tB.data(), (long long)tB.size(),
                             hBias.data(), a.N);
        } else {
            b2g_fill_uniform_f16(tA.data(), (long long)tA.size(), 0, a.seed, 0, a.lo, a.hi);
            b2g_fill_uniform_f16(tB.data(), (long long)tB.size(), 0, a.seed, 1, a.lo, a.hi);
            b2g_fill_uniform_f16(hBias.data(), a.N, 0, a.seed, 2, a.lo, a.hi);
        }
        for (int m = 0; m < a.M; ++m)
            memcpy(&hA[(size_t)m * lda], &tA[(size_t)m * a.K], (size_t)a.K * 2);
        // tB is N x K; in KN mode store its transpose
        for (int n = 0; n < a.N; ++n)
            for (int k = 0; k < a.K; ++k) {
                const uint16_t v = tB[(size_t)n * a.K + k];
                if (a.b_layout == B2G_B_NK) hB[(size_t)n * ldb + k] = v;
                else hB[(size_t)k * ldb + n] = v;
            }
    }
    if (a.gpus != 1 || a.allgather) return run_multi(a, hA, hB, hBias, lda, ldb, ldd);

    void *dA, *dB, *dD, *dRef, *dBias;
    float* dErr;
    CUDA_CHECK(cudaMalloc(&dA, std::max<size_t>(nA, 8) * 2));
    CUDA_CHECK(cudaMalloc(&dB, std::max<size_t>(nB, 8) * 2));
    CUDA_CHECK(cudaMalloc(&dD, std::max<size_t>(nD, 8) * 2));
    CUDA_CHECK(cudaMalloc(&dRef, std::max<size_t>(nD, 8) * 2));
    CUDA_CHECK(cudaMalloc(&dBias, hBias.size() * 2));
    CUDA_CHECK(cudaMalloc(&dErr, sizeof(float)));
    CUDA_CHECK(cudaMemcpy(dA, hA.data(), nA * 2, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(dB, hB.data(), nB * 2, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(dBias, hBias.data(), hBias.size() * 2, cudaMemcpyHostToDevice));
    cudaStream_t stream = 0;

    const double flop = 2.0 * a.M * a.N * a.K;
    double ref_ms = 0, ref_tflops = 0;
    const bool cublas_ok = a.b_layout == B2G_B_NK && lda == a.K;  // the reference call's layout
    if ((a.ref || a.check) && cublas_ok && a.M && a.N && a.K) {
        for (int i = 0; i < a.warmup; ++i)
            if (b2g_cublas_gemm(dA, dB, dRef, a.M, a.N, a.K, stream)) {
                fprintf(stderr, "cuBLAS: %s\n", b2g_last_error());
                return 1;
            }
        cudaEvent_t t0, t1;
        CUDA_CHECK(cudaEventCreate(&t0));
        CUDA_CHECK(cudaEventCreate(&t1));
        CUDA_CHECK(cudaEventRecord(t0, stream));
        for (int i = 0; i < a.iters; ++i) b2g_cublas_gemm(dA, dB, dRef, a.M, a.N, a.K, stream);
        CUDA_CHECK(cudaEventRecord(t1, stream));
        CUDA_CHECK(cudaEventSynchronize(t1));
        float tot = 0;
        CUDA_CHECK(cudaEventElapsedTime(&tot, t0, t1));
        ref_ms = tot / std::max(1, a.iters);
        ref_tflops = flop / (ref_ms * 1e-3) / 1e12;
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
    }

    const bool epi = a.fused || a.unfused;
    printf("# device        : %s  sm_%d%d  %d SMs\n", prop.name, prop.major, prop.minor,
           prop.multiProcessorCount);
    printf("# problem       : M=%d N=%d K=%d  fp16 in / %s acc / fp16 out  (A row-major, B %s)\n",
           a.M, a.N, a.K, a.acc == B2G_ACC_F32 ? "fp32" : "fp16",
           a.b_layout == B2G_B_NK ? "N x K (col-major K x N)" : "K x N row-major");
    printf("# accumulate    : %s\n", a.acc == B2G_ACC_F32 ? "FP32 (tcgen05 kind::f16, F32 D in TMEM)"
                                                          : "FP16 (tcgen05 kind::f16, F16 D in TMEM)");
    printf("# epilogue      : %s\n", a.fused ? "FUSED alpha*acc + bias + ReLU"
                                             : a.unfused ? "UNFUSED bias+ReLU kernel" : "plain store");
    printf("# inputs        : %s\n", a.init_ref ? "reference LCG (seed 12345)" : "seeded uniform");
    printf("# iters         : %d (warmup %d)\n", a.iters, a.warmup);
    if (a.ref && ref_ms > 0) printf("# cuBLAS (SoL)  : %8.3f ms  %7.2f TFLOP/s\n", ref_ms, ref_tflops);
    printf("\n");
    printf("%-6s %-12s %-8s %6s %5s %5s %7s %6s %6s %10s %9s %8s %s\n", "tile", "CTA", "layout",
           "stages", "grp", "thr", "reg/thr", "smem", "CTA/SM", "ms", "TFLOP/s", "%SoL", "maxrel");
    printf("%s\n", std::string(118, '-').c_str());

    struct Job { int tile, layout, stages, group; };
    std::vector<Job> jobs;
    if (a.sweep) {
        for (int s = 2; s <= 8; ++s) jobs.push_back({a.tile, a.layout, s, a.group});
    } else if (a.gsweep) {
        for (int g : {1, 2, 4, 8, 16}) jobs.push_back({a.tile, a.layout, a.stages, g});
    } else {
        jobs.push_back({a.tile, a.layout, a.stages, a.group});
    }

    int rc_all = 0;
    for (const Job& j : jobs) {
        auto skip = [&](const char* why) {
            printf("%-6d %-12s %-8s %6d %5d %5s %7s %6s %6s %10s %9s %8s  SKIP: %s\n", j.tile,
                   tile_name(j.tile), "sw128", j.stages, j.group, "-", "-", "-", "-", "-", "-",
                   "-", why);
        };
        if (j.layout != 2) {
            skip("layout not applicable on sm_100a (TMA writes the 128B-swizzled UMMA layout)");
            continue;
        }
        int thr = 0, regs = 0, smem = 0, occ = 0, tmem = 0, st_used = 0;
        if (b2g_config_info(j.tile, j.stages, &thr, &regs, &smem, &occ, &tmem, &st_used)) {
            skip(b2g_last_error());
            continue;
        }
        CUDA_CHECK(cudaMemset(dD, 0, std::max<size_t>(nD, 8) * 2));
        auto launch = [&]() -> int {
            const int epi = a.fused ? B2G_EPI_BIAS_RELU : B2G_EPI_NONE;
            int rc = a.splits < 0
                         ? b2g_gemm(dA, dB, dD, a.fused ? dBias : nullptr, a.M, a.N, a.K, lda, ldb,
                                    ldd, a.b_layout, a.acc, epi, 1.0f, j.tile, j.stages, j.group,
                                    stream)
                         : b2g_gemm_splitk(dA, dB, dD, a.fused ? dBias : nullptr, a.M, a.N, a.K,
                                           lda, ldb, ldd, a.b_layout, a.acc, epi, 1.0f, j.tile,
                                           j.stages, j.group, a.splits, stream);
            if (rc == B2G_OK && a.unfused)
                rc = b2g_bias_relu(dD, dBias, a.M, a.N, ldd, 1.0f, stream);
            return rc;
        };
        int rc = B2G_OK;
        for (int i = 0; i < a.warmup && rc == B2G_OK; ++i) rc = launch();
        if (rc == B2G_OK) rc = b2g_sync_status(stream);
        if (rc != B2G_OK) {
            skip(b2g_last_error());
            rc_all = 1;
            continue;
        }
        int used_splits = 1;
        if (a.warmup > 0) b2g_last_launch(nullptr, &thr, nullptr, &st_used, nullptr, &used_splits);
        cudaEvent_t t0, t1;
        CUDA_CHECK(cudaEventCreate(&t0));
        CUDA_CHECK(cudaEventCreate(&t1));
        double ms = 0, tflops = 0;
        if (a.soak > 0) {
            printf("# soak %.0f s, window %.1f s -- columns are parseable CSV after 'SOAK,'\n",
                   a.soak, a.window);
            printf("SOAK,elapsed_s,window_ms,iters,tflops,ms_per_iter\n");
            fflush(stdout);
            const double wall0 = now_s();
            double best = 0, worst = 1e30, sum_flop = 0, sum_s = 0;
            int nwin = 0;
            while (now_s() - wall0 < a.soak) {
                int n = 0;
                CUDA_CHECK(cudaEventRecord(t0, stream));
                const double ws = now_s();
                do {
                    launch();
                    ++n;
                    if ((n & 7) == 0) CUDA_CHECK(cudaStreamSynchronize(stream));
                } while (now_s() - ws < a.window);
                CUDA_CHECK(cudaEventRecord(t1, stream));
                CUDA_CHECK(cudaEventSynchronize(t1));
                float wms = 0;
                CUDA_CHECK(cudaEventElapsedTime(&wms, t0, t1));
                const double tf = flop * n / (wms * 1e-3) / 1e12;
                printf("SOAK,%.2f,%.2f,%d,%.3f,%.4f\n", now_s() - wall0, wms, n, tf, wms / n);
                fflush(stdout);
                best = std::max(best, tf);
                worst = std::min(worst, tf);
                sum_flop += flop * n;
                sum_s += wms * 1e-3;
                ++nwin;
            }
            const double avg = sum_flop / sum_s / 1e12;
            printf("# soak summary: windows=%d  avg=%.2f  max=%.2f  min=%.2f TFLOP/s  spread=%.1f%%\n",
                   nwin, avg, best, worst, 100.0 * (best - worst) / best);
            ms = sum_s * 1e3 / (sum_flop / flop);
            tflops = avg;
        } else {
            CUDA_CHECK(cudaEventRecord(t0, stream));
            for (int i = 0; i < a.iters; ++i) launch();
            CUDA_CHECK(cudaEventRecord(t1, stream));
            CUDA_CHECK(cudaEventSynchronize(t1));
            float tot = 0;
            CUDA_CHECK(cudaEventElapsedTime(&tot, t0, t1));
            ms = tot / std::max(1, a.iters);
            tflops = flop / (ms * 1e-3) / 1e12;
        }
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        rc = b2g_sync_status(stream);
        if (rc != B2G_OK) {
            skip(b2g_last_error());
            rc_all = 1;
            continue;
        }

        double maxrel = -1, cpurel = -1, frob = -1;
        int wm = -1, wn = -1;
        if (a.check && !epi && cublas_ok && ref_ms > 0) {
            b2g_max_rel_diff(dD, dRef, nD, dErr, stream);
            float e = 0;
            CUDA_CHECK(cudaMemcpy(&e, dErr, sizeof e, cudaMemcpyDeviceToHost));
            maxrel = e;
        }
        if (a.cpu > 0 || a.frob > 0) {
            std::vector<uint16_t> hD(nD);
            CUDA_CHECK(cudaMemcpy(hD.data(), dD, nD * 2, cudaMemcpyDeviceToHost));
            if (a.cpu > 0)
                cpurel = spot_check(hA, lda, hB, ldb, a.b_layout, hD, ldd, hBias, a.M, a.N, a.K,
                                    a.cpu, epi, 1.0f, &wm, &wn);
            if (a.frob > 0)
                frob = frobenius_rows(hA, lda, hB, ldb, a.b_layout, hD, ldd, hBias, a.M, a.N, a.K,
                                      a.frob, epi, 1.0f);
        }
        char errbuf[32], solbuf[16];
        if (maxrel < 0) snprintf(errbuf, sizeof errbuf, "-");
        else snprintf(errbuf, sizeof errbuf, "%.2e%s", maxrel, maxrel < 3e-2 ? " OK" : " FAIL");
        if (a.ref && ref_tflops > 0) snprintf(solbuf, sizeof solbuf, "%.1f%%", 100.0 * tflops / ref_tflops);
        else snprintf(solbuf, sizeof solbuf, "-");
        printf("%-6d %-12s %-8s %6d %5d %5d %7d %6d %6d %10.3f %9.2f %8s %s", j.tile,
               tile_name(j.tile), "sw128", st_used, j.group, thr, regs, smem, occ, ms, tflops,
               solbuf, errbuf);
        if (cpurel >= 0)
            printf("  cpu=%.2e%s(worst m=%d n=%d)", cpurel, cpurel < 3e-2 ? " OK " : " FAIL ", wm, wn);
        if (frob >= 0) printf("  frob=%.2e", frob);
        double kmhz = 0, kus = 0;
        if (b2g_kernel_clock(&kmhz, &kus) == B2G_OK) printf("  sm_mhz=%.0f", kmhz);
        printf("  splits=%d\n", used_splits);
        if (a.json)
            printf("{\"M\": %d, \"N\": %d, \"K\": %d, \"tile\": %d, \"stages\": %d, \"group\": %d, "
                   "\"acc\": \"%s\", \"ms\": %.5f, \"tflops\": %.3f, \"cublas_tflops\": %.3f, "
                   "\"maxrel_vs_cublas\": %.3e, \"cpu_maxrel\": %.3e, \"frob_rel\": %.3e, "
                   "\"splits\": %d, \"sm_mhz\": %.0f}\n",
                   a.M, a.N, a.K, j.tile, st_used, j.group, a.acc == B2G_ACC_F32 ? "f32" : "f16", ms,
                   tflops, ref_tflops, maxrel, cpurel, frob, used_splits, kmhz);
        fflush(stdout);
    }
    cudaFree(dA); cudaFree(dB); cudaFree(dD); cudaFree(dRef); cudaFree(dBias); cudaFree(dErr);
    return rc_all;
}
