// gemm_sm100_2cta.cuh -- persistent FP16 GEMM on 2-CTA clusters (tcgen05 cta_group::2).
//
// A cluster of two CTAs on two SMs computes one 256 x 256 output tile with UMMA
// 256 x 256 x 16 instructions issued by the even ("leader") CTA. Each CTA stages only its
// own half of the operands in shared memory -- 128 rows of A and 128 rows of B per k-block
// (32 KiB per stage instead of 48 KiB for a 128 x 256 tile on one SM) -- and the tensor
// core reads both CTAs' halves. Every CTA keeps its 128 rows of the 256 x 256 accumulator
// in its own TMEM, double-buffered (2 x 256 columns). No TMA multicast is used: each CTA
// loads its halves itself (this code also runs on multi-GPU jobs).
//
// Roles (192 threads per CTA):
//   warp 0, one thread, both CTAs: TMA producer. Waits for its stage's `empty` barrier,
//     then loads its A half (128 x 64) and B half (128 x 64). Both CTAs' loads complete
//     on the LEADER's `full` barrier, which the leader's producer armed with the pair's
//     total byte count (2 x 32 KiB).
//   warp 1, one thread, leader only: MMA issuer. Waits for `full` (both halves landed),
//     issues 4 x tcgen05.mma.cta_group::2, then a multicast tcgen05.commit that arrives on
//     the `empty` barrier of the same stage in both CTAs. After the last k-block, a
//     multicast commit on `tmem_full[buf]` of both CTAs.
//   warps 2-5, both CTAs: epilogue of this CTA's 128 rows (same as the 1-CTA kernel),
//     then one arrive per warp on the leader's `tmem_empty[buf]` (count 8).
// Barrier waits are cluster-scope acquires (their arrivals come from the peer SM).
#pragma once

#include "gemm_sm100.cuh"

namespace b2g {

constexpr int kPairBM = 256;                       // pair tile rows (128 per CTA)
constexpr int kPairBN = 256;                       // pair tile columns = UMMA N
constexpr uint32_t kHalfBytes = 128 * kBK * 2;     // one operand half per k-block: 16 KiB
constexpr uint32_t kPairStageBytes = 2 * kHalfBytes;  // per CTA: A half + B half
constexpr uint32_t kPairTmemCols = 2 * kPairBN;    // double-buffered accumulator

constexpr size_t gemm2_smem_bytes(int stages) {
    return 1024 + (size_t)stages * kPairStageBytes + sizeof(SmemCtl);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_sm100_2cta(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    extern __shared__ uint8_t smem_dyn[];
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    const uint32_t sA = raw + pad;
    const uint32_t sB = sA + (uint32_t)p.stages * kHalfBytes;
    SmemCtl* ctl =
        reinterpret_cast<SmemCtl*>(smem_dyn + pad + (size_t)p.stages * kPairStageBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster_id = blockIdx.x >> 1, num_clusters = gridDim.x >> 1;
    const uint32_t full0 = smem_u32(&ctl->full[0]);
    const uint32_t empty0 = smem_u32(&ctl->empty[0]);
    const uint32_t tfull0 = smem_u32(&ctl->tmem_full[0]);
    const uint32_t tempty0 = smem_u32(&ctl->tmem_empty[0]);
    const uint32_t drain = smem_u32(&ctl->drain);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);   // only the leader's copy is used
            mbar_init(empty0 + 8 * s, 1);  // one multicast commit per use
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 8);  // 4 epilogue warps x 2 CTAs (leader's copy)
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
        tmem_alloc<2>(smem_u32(&ctl->tmem_base), kPairTmemCols);
        tmem_relinquish<2>();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // peer barriers are initialised before anyone signals them
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;
    volatile int* abort_flag = &ctl->abort;
    volatile int* no_abort = &ctl->never;
    const uint32_t full0_leader = mapa_shared(full0, 0);
    const uint32_t tempty0_leader = mapa_shared(tempty0, 0);

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------ TMA producer ------------------------------
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitProducer};
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = cluster_id; t < p.num_tiles && ok; t += num_clusters) {
                int tm, tn;
                tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
                const int m0 = tm * kPairBM + (int)rank * 128;
                const int n0 = tn * kPairBN + (int)rank * 128;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait<true>(empty0 + 8 * stage, phase ^ 1u, w)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(full0 + 8 * stage, 2 * kPairStageBytes);
                    const uint32_t fb = full0_leader + 8 * stage;
                    tma_load_2d_pair(sA + stage * kHalfBytes, &tmA, fb, kb * kBK, m0);
                    tma_load_2d_pair(sB + stage * kHalfBytes, &tmB, fb, kb * kBK, n0);
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // unwind: give loads still in flight time to land before the CTA exits
                const uint64_t t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 200000ull) {
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ------------------------------- MMA issuer -------------------------------
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitMma};
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int t = cluster_id; t < p.num_tiles && ok; t += num_clusters, ++it) {
                const int buf = it & 1;
                const uint32_t use = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait<true>(tempty0 + 8 * buf, use ^ 1u, w)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kPairBN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait<true>(full0 + 8 * stage, phase, w)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sA + stage * kHalfBytes;
                    const uint32_t b0 = sB + stage * kHalfBytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        const uint64_t ad = sdesc_sw128(a0 + 32u * k, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b0 + 32u * k, 16, 1024);
                        mma_f16_ss<2>(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit_pair(empty0 + 8 * stage, 0x3);  // frees the stage in both CTAs
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit_pair(tfull0 + 8 * buf, 0x3);  // accumulator final in both CTAs
            }
            const WaitCtx wd{p.timeout_ns, no_abort, kErrWaitDrain};
            mma_commit_2(drain);
            mbar_wait<true>(drain, 0, wd);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------------
        const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitEpilogue};
        const int q = warp & 3;
        int it = 0;
        for (int t = cluster_id; t < p.num_tiles; t += num_clusters, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1) & 1u;
            const bool ok = mbar_wait<true>(tfull0 + 8 * buf, use, w);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            int tm, tn;
            tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
            const int row = tm * kPairBM + (int)rank * 128 + q * 32 + lane;
            const uint32_t tbase =
                tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kPairBN);
#pragma unroll 1
            for (int c = 0; c < kPairBN; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tbase + (uint32_t)c, r);
                tmem_ld_wait();
                store_row_chunk32(p, row, tn * kPairBN + c, r);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty0_leader + 8 * buf);
        }
    }

    // teardown: no CTA may leave while its peer can still signal its barriers or while
    // MMAs may still write TMEM (the leader drained them above)
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<2>(tmem_base, kPairTmemCols);
    }
}

}  // namespace b2g
