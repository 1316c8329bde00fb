// gemm_sm100.cuh -- persistent, warp-specialised FP16 GEMM for sm_100a (one CTA per tile).
//
// Replaces the reference's gemm_kernel (src/gemm_bench.cu:213-399). The reference stages
// operands with per-thread cp.async into a STAGES-deep ring, moves them to registers with
// ldmatrix and multiplies with warp-level mma.sync, one CTA per output tile. Here:
//
//   warp 0 (1 thread)  TMA producer: for every k-block, wait for a free stage, then two
//                      cp.async.bulk.tensor loads (A 128x64, B BNx64, 128-byte swizzle)
//                      whose bytes complete the stage's `full` mbarrier.
//   warp 1 (1 thread)  MMA issuer: allocates TMEM (2 x BN columns: a double-buffered
//                      accumulator), waits for `full`, issues 4 tcgen05.mma (K = 16 each)
//                      reading both operands from shared memory, and tcgen05.commit's the
//                      stage's `empty` barrier; after the last k-block it commits
//                      `tmem_full[buf]`.
//   warps 2-5          epilogue: wait for `tmem_full[buf]`, tcgen05.ld 32 columns at a time
//                      (warp w reads TMEM lanes 32*(w%4)..+31 = tile rows), apply the
//                      optional alpha*acc + bias + ReLU, round to FP16 (RN, as
//                      __floats2half2_rn in the reference) and store; then arrive on
//                      `tmem_empty[buf]` so the MMA warp can reuse that accumulator.
//
// The grid is persistent (<= one CTA per SM); CTA b processes linear tiles b, b + grid, ...
// mapped by tile_coord (the reference's grouped rasterization). Because the accumulator is
// double-buffered, the epilogue of tile i overlaps the mainloop of tile i + 1.
//
// M, N and K edges: TMA zero-fills out-of-range rows and k columns of a box, so partial
// tiles need no special mainloop; the epilogue skips rows >= M and columns >= N.
#pragma once

#include <cuda_fp16.h>

#include "sm100_ptx.cuh"
#include "tile_sched.h"

namespace b2g {

struct GemmParams {
    int M, N, K;
    int tiles_m, tiles_n, num_tiles, num_kb;
    int group, stages;
    uint32_t idesc;
    int acc_f16;   // accumulator is F16: each 32-bit TMEM column holds one value in bits 0..15
    int epilogue;  // 0 plain store, 1 alpha*acc + bias + ReLU
    float alpha;
    const __half* bias;
    __half* D;
    long long ldd;
    int d_vec;       // 16-byte vector stores allowed (D 16-byte aligned and ldd % 8 == 0)
    int b_mn_major;  // B is K x N (MN-major) in global memory
    unsigned long long timeout_ns;
};

constexpr int kBM = 128;      // rows of A per CTA (UMMA M for cta_group::1)
constexpr int kBK = 64;       // k-block: one 128-byte swizzle row of FP16
constexpr int kUmmaK = 16;    // K of one kind::f16 MMA
constexpr int kMaxStages = 8;
constexpr int kThreads = 192; // producer warp, MMA warp, 4 epilogue warps
constexpr uint32_t kAStageBytes = kBM * kBK * 2;  // 16 KiB

template <int BN>
struct TileTraits {
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, step 64");
    static constexpr uint32_t kBStageBytes = BN * kBK * 2;
    static constexpr uint32_t kStageBytes = kAStageBytes + kBStageBytes;
    static constexpr uint32_t kTmemCols = 2 * BN;  // power of two for BN in {128, 256}
};

struct SmemCtl {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    int never;  // stays 0: lets teardown waits ignore `abort` and use only their time limit
};

template <int BN>
constexpr size_t gemm_smem_bytes(int stages) {
    return 1024 /* alignment slack */ + (size_t)stages * TileTraits<BN>::kStageBytes +
           sizeof(SmemCtl);
}

__device__ __forceinline__ float acc_value(uint32_t raw, int acc_f16) {
    return acc_f16 ? __half2float(__ushort_as_half((unsigned short)(raw & 0xFFFFu)))
                   : __uint_as_float(raw);
}

// Epilogue for 32 consecutive columns [col, col + 32) of one output row.
__device__ __forceinline__ void store_row_chunk32(const GemmParams& p, int row, int col,
                                                  const uint32_t (&r)[32]) {
    if (row >= p.M || col >= p.N) return;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = acc_value(r[j], p.acc_f16);
    if (p.epilogue) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float x;
            if (p.bias != nullptr) {
                const int n = col + j < p.N ? col + j : p.N - 1;
                x = fmaf(v[j], p.alpha, __half2float(p.bias[n]));
            } else {
                x = v[j] * p.alpha;
            }
            v[j] = x > 0.f ? x : 0.f;
        }
    }
    __half* dst = p.D + (size_t)row * (size_t)p.ldd + col;
    if (p.d_vec && col + 32 <= p.N) {
        uint32_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            __half2 t = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            h[j] = *reinterpret_cast<uint32_t*>(&t);
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        d4[0] = make_uint4(h[0], h[1], h[2], h[3]);
        d4[1] = make_uint4(h[4], h[5], h[6], h[7]);
        d4[2] = make_uint4(h[8], h[9], h[10], h[11]);
        d4[3] = make_uint4(h[12], h[13], h[14], h[15]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (col + j < p.N) dst[j] = __float2half_rn(v[j]);
    }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sm100_1cta(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using TT = TileTraits<BN>;
    extern __shared__ uint8_t smem_dyn[];
    // stage buffers must be 1024-byte aligned (128-byte swizzle atoms, base offset 0)
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    const uint32_t sA = raw + pad;
    const uint32_t sB = sA + (uint32_t)p.stages * kAStageBytes;
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem_dyn + pad + (size_t)p.stages * TT::kStageBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(&ctl->full[0]);
    const uint32_t empty0 = smem_u32(&ctl->empty[0]);
    const uint32_t tfull0 = smem_u32(&ctl->tmem_full[0]);
    const uint32_t tempty0 = smem_u32(&ctl->tmem_empty[0]);
    const uint32_t drain = smem_u32(&ctl->drain);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 4);  // one arrive per epilogue warp
        }
        mbar_init(drain, 1);
        ctl->abort = 0;
        ctl->never = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc<1>(smem_u32(&ctl->tmem_base), TT::kTmemCols);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;
    volatile int* abort_flag = &ctl->abort;
    volatile int* no_abort = &ctl->never;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------ TMA producer ------------------------------
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitProducer};
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                int tm, tn;
                tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
                const int m0 = tm * kBM, n0 = tn * BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, w)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_arrive_expect_tx(fb, TT::kStageBytes);
                    tma_load_2d(sA + stage * kAStageBytes, &tmA, fb, kb * kBK, m0);
                    tma_load_2d(sB + stage * TT::kBStageBytes, &tmB, fb, kb * kBK, n0);
                    ++issued;
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // unwind: wait (bounded) until the loads still in flight have landed
                const WaitCtx wd{p.timeout_ns, no_abort, kErrWaitDrain};
                const long long outstanding = issued < p.stages ? issued : p.stages;
                for (long long i = 0; i < outstanding; ++i) {
                    if (stage == 0) {
                        stage = p.stages - 1;
                        phase ^= 1u;
                    } else {
                        --stage;
                    }
                    if (!mbar_wait(full0 + 8 * stage, phase, wd)) break;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------- MMA issuer -------------------------------
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitMma};
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++it) {
                const int buf = it & 1;
                const uint32_t use = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(tempty0 + 8 * buf, use ^ 1u, w)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, w)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sA + stage * kAStageBytes;
                    const uint32_t b0 = sB + stage * TT::kBStageBytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        const uint64_t ad = sdesc_sw128(a0 + 32u * k, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b0 + 32u * k, 16, 1024);
                        mma_f16_ss<1>(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(empty0 + 8 * stage);  // frees the stage once these MMAs retire
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * buf);  // accumulator `buf` is final
            }
            // drain: nothing may still read shared memory or write TMEM at teardown
            const WaitCtx wd{p.timeout_ns, no_abort, kErrWaitDrain};
            mma_commit(drain);
            mbar_wait(drain, 0, wd);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------------
        const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitEpilogue};
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int it = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1) & 1u;
            const bool ok = mbar_wait(tfull0 + 8 * buf, use, w);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            int tm, tn;
            tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
            const int row = tm * kBM + q * 32 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tbase + (uint32_t)c, r);
                tmem_ld_wait();
                store_row_chunk32(p, row, tn * BN + c, r);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
        }
    }

    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, TT::kTmemCols);
    }
}

}  // namespace b2g
