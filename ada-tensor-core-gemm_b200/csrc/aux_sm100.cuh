// aux_sm100.cuh -- small kernels around the GEMM: the device-side max relative difference,
// the unfused bias+ReLU epilogue, the K == 0 epilogue fill, the HBM stream probe, the
// all-gather push of D panels to peer devices and the bounded-wait self-test. All are bandwidth-bound elementwise kernels with grid-stride
// loops over 16-byte (or 2-byte at ragged edges) accesses.
#pragma once

#include <cuda_fp16.h>

#include "b2g_internal.h"
#include "sm100_ptx.cuh"

namespace b2g {

// max over i of |x_i - y_i| / max(1, |y_i|) into *out (FP32 bits, atomicMax; all values are
// non-negative so the integer order of the bits is the float order). Same metric as the
// reference's max_rel_diff (src/gemm_bench.cu:648-664).
__global__ void __launch_bounds__(256) max_rel_diff_kernel(const __half* __restrict__ x,
                                                           const __half* __restrict__ y,
                                                           size_t n, float* out) {
    float m = 0.f;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)blockDim.x * gridDim.x) {
        const float a = __half2float(x[i]), b = __half2float(y[i]);
        const float d = fabsf(a - b) / fmaxf(1.f, fabsf(b));
        m = fmaxf(m, d != d ? __int_as_float(0x7f800000) : d);  // NaN counts as infinitely wrong
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float r = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = fmaxf(r, red[w]);
        atomicMax(reinterpret_cast<int*>(out), __float_as_int(r));
    }
}

// D[m, n] = relu(alpha * D[m, n] + bias[n]), FP32 math, FP16 round-to-nearest store.
// The reference's --unfused path (src/gemm_bench.cu:401-408) on a row-major D with ldd.
__global__ void __launch_bounds__(256) bias_relu_kernel(__half* D, const __half* __restrict__ bias,
                                                        int M, int N, long long ldd, float alpha) {
    const size_t total = (size_t)M * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)blockDim.x * gridDim.x) {
        const size_t m = i / (size_t)N, n = i - m * (size_t)N;
        __half* d = D + m * (size_t)ldd + n;
        float v = __half2float(*d);
        // multiply, then add (two roundings), as src/gemm_bench.cu:405-406 compiles
        v = __fmul_rn(v, alpha);
        if (bias) v = __fadd_rn(v, __half2float(bias[n]));
        *d = __float2half_rn(v > 0.f ? v : 0.f);
    }
}

// K == 0: the accumulator is zero, so D = epilogue(0) = relu(bias) (or 0).
__global__ void __launch_bounds__(256) zero_k_fill_kernel(__half* D, const __half* __restrict__ bias,
                                                          int M, int N, long long ldd,
                                                          int epilogue) {
    const size_t total = (size_t)M * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)blockDim.x * gridDim.x) {
        const size_t m = i / (size_t)N, n = i - m * (size_t)N;
        float v = 0.f;
        if (epilogue && bias) {
            v = __half2float(bias[n]);
            v = v > 0.f ? v : 0.f;
        }
        D[m * (size_t)ldd + n] = __float2half_rn(v);
    }
}

// Streaming copy for the HBM roof: 16-byte loads and stores, 4 in flight per thread.
// n16 = number of 16-byte words. Replaces bw_kernel (src/device_query.cu:170-175).
__global__ void __launch_bounds__(512) hbm_copy_kernel(const uint4* __restrict__ src,
                                                       uint4* __restrict__ dst, size_t n16) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n16; i += 4 * stride) {
        const uint4 a = __ldcs(src + i);
        const uint4 b = __ldcs(src + i + stride);
        const uint4 c = __ldcs(src + i + 2 * stride);
        const uint4 d = __ldcs(src + i + 3 * stride);
        __stcs(dst + i, a);
        __stcs(dst + i + stride, b);
        __stcs(dst + i + 2 * stride, c);
        __stcs(dst + i + 3 * stride, d);
    }
    for (; i < n16; i += stride) __stcs(dst + i, __ldcs(src + i));
}

// Failure-detection self-test: wait on an mbarrier that nothing arrives at, bounded by
// `timeout_ns`; the wait records kErrWaitSelftest in the status word and returns.
// Destinations of one device's all-gather push: its own full D and the peers' (same rows);
// kMaxGatherDst (8) comes from b2g_internal.h.
struct GatherDst {
    int n;
    __half* d[kMaxGatherDst];
};

// Copy `rows` x `n8` 16-byte groups of a D panel (pitch ldd elements) to every destination
// with the same pitch: each group is read once from HBM and stored to all n destinations
// (peer ones over NVLink), four groups per thread in flight. Blocks stride over rows,
// threads over a row's groups.
__global__ void __launch_bounds__(256) allgather_push_kernel(const __half* __restrict__ src,
                                                             int rows, int n8, long long ldd,
                                                             GatherDst dst) {
    const int bs = blockDim.x;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const size_t row = (size_t)r * (size_t)ldd;
        const uint4* srow = reinterpret_cast<const uint4*>(src + row);
        for (int c0 = threadIdx.x; c0 < n8; c0 += 4 * bs) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + u * bs < n8) v[u] = __ldcs(srow + c0 + u * bs);
#pragma unroll
            for (int q = 0; q < kMaxGatherDst; ++q) {  // constant indices into the parameters
                if (q < dst.n) {
                    uint4* drow = reinterpret_cast<uint4*>(dst.d[q] + row);
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (c0 + u * bs < n8) st_global_cs_v4(drow + c0 + u * bs, v[u]);
                }
            }
        }
    }
}

__global__ void selftest_wait_kernel(unsigned long long timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(smem_u32(&bar), 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const WaitCtx w{timeout_ns, &abort_flag, kErrWaitSelftest};
        mbar_wait(smem_u32(&bar), 0, w);  // phase 0 never completes
    }
    __syncthreads();
}

}  // namespace b2g
