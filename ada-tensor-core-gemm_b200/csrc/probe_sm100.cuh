// probe_sm100.cuh -- tcgen05 issue-rate probe: the achievable dense tensor throughput per SM.
//
// Replaces the reference's mma_probe (src/device_query.cu:48-138), which times NACC chains
// of register-resident mma.sync with clock64(). On sm_100 the tensor core is driven by a
// single thread issuing tcgen05.mma with both operands in shared memory and the accumulator
// in TMEM, so the probe does exactly that: one CTA per SM, operand tiles written once into
// 128-byte-swizzled shared memory, then `iters` back-to-back MMAs into one accumulator,
// a tcgen05.commit, a bounded wait for completion, and the clock64() delta. Nothing in the
// loop touches memory, so the only limit is the tensor pipe. The cta_group::2 form measures
// the pair MMA that the 2-CTA GEMM kernels issue (UMMA M = 256 over two SMs).
#pragma once

#include "sm100_ptx.cuh"

namespace b2g {

enum { kProbeF16F32 = 0, kProbeF16F16 = 1, kProbeI8 = 2, kProbeE4M3 = 3 };

// Instruction descriptor for the probe kinds: D format (bits 4..5: F16 0, F32 1, S32 2),
// A/B formats (bits 7..9 / 10..12: kind::f16 F16 = 0; kind::i8 signed = 1;
// kind::f8f6f4 E4M3 = 0), both operands K-major, N >> 3 at 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t idesc_probe(int kind, int m, int n) {
    const uint32_t c = kind == kProbeF16F16 ? 0u : (kind == kProbeI8 ? 2u : 1u);
    const uint32_t ab = kind == kProbeI8 ? 1u : 0u;
    return (c << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

__host__ __device__ constexpr int probe_mma_k(int kind) {
    return (kind == kProbeI8 || kind == kProbeE4M3) ? 32 : 16;
}

constexpr int kProbeThreads = 128;
constexpr uint32_t kProbeABytes = 128 * 128;  // 128 rows x 128 B
constexpr uint32_t kProbeBBytes = 256 * 128;  // up to 256 rows x 128 B
// more than half of the SM's shared memory, so exactly one probe CTA is resident per SM
constexpr size_t kProbeSmem = 128 * 1024;
static_assert(kProbeSmem >= 1024 + kProbeABytes + kProbeBBytes + 64, "probe smem too small");

// Fill this CTA's operand tiles with small values, so no accumulator overflows over
// thousands of MMAs: F16 2^-8 (0x1C00), S8 1, E4M3 2^-4 (0x18).
template <int KIND>
__device__ __forceinline__ void probe_fill(uint8_t* base) {
    const uint32_t word =
        KIND == kProbeI8 ? 0x01010101u : (KIND == kProbeE4M3 ? 0x18181818u : 0x1C001C00u);
    uint32_t* w32 = reinterpret_cast<uint32_t*>(base);
    for (uint32_t i = threadIdx.x; i < (kProbeABytes + kProbeBBytes) / 4; i += blockDim.x)
        w32[i] = word;
    fence_proxy_async_smem();
}

// `iters` back-to-back MMAs into one accumulator (the k offset cycles through the 128-byte
// row so consecutive MMAs read different operand bytes, as a GEMM's K steps do).
template <int KIND, int CG>
__device__ __forceinline__ void probe_issue(uint32_t tmem, uint32_t sA, uint32_t sB,
                                            uint32_t idesc, int iters) {
    for (int i = 0; i < iters; ++i) {
        const uint32_t koff = 32u * (uint32_t)(i & 3);
        const uint64_t ad = sdesc_sw128(sA + koff, 16, 1024);
        const uint64_t bd = sdesc_sw128(sB + koff, 16, 1024);
        const uint32_t acc = i > 0 ? 1u : 0u;
        if constexpr (KIND == kProbeI8)
            mma_i8_ss<CG>(tmem, ad, bd, idesc, acc);
        else if constexpr (KIND == kProbeE4M3)
            mma_f8_ss<CG>(tmem, ad, bd, idesc, acc);
        else
            mma_f16_ss<CG>(tmem, ad, bd, idesc, acc);
    }
}

template <int KIND>
__global__ void __launch_bounds__(kProbeThreads, 1)
    probe_tcgen05_kernel(uint32_t idesc, int iters, long long* cycles,
                         unsigned long long timeout_ns) {
    extern __shared__ uint8_t smem_dyn[];
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    uint8_t* base = smem_dyn + pad;
    const uint32_t sA = raw + pad, sB = sA + kProbeABytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + kProbeABytes + kProbeBBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    int* abort_flag = reinterpret_cast<int*>(bar + 2);

    probe_fill<KIND>(base);
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x < 32) {
        tmem_alloc<1>(smem_u32(tmem_slot), 256);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (threadIdx.x == 0) {
        const WaitCtx w{timeout_ns, abort_flag, kErrWaitProbe};
        const long long t0 = clock64();
        probe_issue<KIND, 1>(tmem, sA, sB, idesc, iters);
        mma_commit(smem_u32(bar));
        const bool ok = mbar_wait(smem_u32(bar), 0, w);
        const long long t1 = clock64();
        cycles[blockIdx.x] = ok ? (t1 - t0) : -1;
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc_fence_after();
        tmem_dealloc<1>(tmem, 256);
    }
}

// cta_group::2 form: a 2-CTA cluster on two SMs, the pair MMA (UMMA M = 256) issued by the
// even CTA. As in the pair GEMM kernel, each CTA holds its own 128 rows of A and N / 2 rows of
// B at the same shared-memory offsets and its own 128 accumulator lanes in TMEM; the leader's
// clock64 delta covers the pair's `iters` MMAs, so FLOP per clock per SM is half the pair's.
// cycles[] is indexed by cluster.
template <int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kProbeThreads, 1)
    probe_tcgen05_pair_kernel(uint32_t idesc, int iters, long long* cycles,
                              unsigned long long timeout_ns) {
    extern __shared__ uint8_t smem_dyn[];
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    uint8_t* base = smem_dyn + pad;
    const uint32_t sA = raw + pad, sB = sA + kProbeABytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + kProbeABytes + kProbeBBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    int* abort_flag = reinterpret_cast<int*>(bar + 2);
    const bool leader = cluster_ctarank() == 0;

    probe_fill<KIND>(base);
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x < 32) {
        tmem_alloc<2>(smem_u32(tmem_slot), 256);
        tmem_relinquish<2>();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' operands, barriers and TMEM are ready
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (leader && threadIdx.x == 0) {
        const WaitCtx w{timeout_ns, abort_flag, kErrWaitProbe};
        const long long t0 = clock64();
        probe_issue<KIND, 2>(tmem, sA, sB, idesc, iters);
        mma_commit_2(smem_u32(bar));
        const bool ok = mbar_wait(smem_u32(bar), 0, w);
        const long long t1 = clock64();
        cycles[blockIdx.x >> 1] = ok ? (t1 - t0) : -1;
    }
    // no CTA frees its TMEM or leaves while the pair's MMAs may still use its half
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (threadIdx.x < 32) {
        tc_fence_after();
        tmem_dealloc<2>(tmem, 256);
    }
}

}  // namespace b2g
