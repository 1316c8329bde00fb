// gemm_sm100_swap.cuh -- decode-shaped GEMMs (small M) with the operand roles swapped.
//
// The reference's kernel keeps 0.4-44% of its square-GEMM throughput at M = 1..128 with
// N = K = 4096 (docs/RESULTS.md:249-265): a 128-row tile computes mostly padding. Here the
// UMMA's 128-row side is filled by 128 rows of B (128 columns of D) and the small M becomes
// the UMMA N (MT = 16, 32 or 64 rows of A): each CTA computes D^T for a 128-column x MT-row
// block, D^T = B_tile . A_tile^T, with both operands K-major exactly as they lie in memory
// (B: N x K row-major, A: M x K row-major). MT is chosen so the grid has ~one CTA per SM
// without split-K.
//
// Roles as in gemm_sm100_1cta: warp 0 TMA producer (B box 128 rows, A box MT rows per
// 64-wide k-block), warp 1 MMA issuer (UMMA 128 x MT x 16, double-buffered accumulator of
// 2 x MT TMEM columns), warps 2-5 epilogue (4 warps, one per TMEM lane quarter). In TMEM, lane = column n of D and TMEM column j =
// row m0 + j of D, so each thread holds a column of the output block: it converts its MT
// values (alpha, bias[n], ReLU, FP16) and stores them row by row -- for every m the 32 lanes
// of a warp write 32 consecutive columns (64 contiguous bytes). No staging, no TMA store.
//
// With N = 4096 the 128-row blocks give only 32 CTAs. The narrow form (NARROW) takes ~N / SMs
// rows of B per CTA instead (32 at N = 4096: 128 CTAs), several k-blocks per ring stage, and
// streams every CTA's rows over the whole K range: all SMs read B at once and no split-K
// reduction follows the mainloop. Measured at decode shapes it stays behind the 128 x 128
// tiles with cluster split-K (M = 1: 12.0 vs 11.6 us), so b2g_gemm never picks it on its own.
#pragma once

#include "gemm_sm100.cuh"

namespace b2g {

template <int MT>
struct SwapTraits {
    static_assert(MT == 16 || MT == 32 || MT == 64, "MT = 16, 32 or 64");
    static constexpr uint32_t kBStageBytes = 128 * kBK * 2;  // 128 rows of B: 16 KiB
    static constexpr uint32_t kAStageBytes = MT * kBK * 2;   // MT rows of A
    static constexpr uint32_t kStageBytes = kBStageBytes + kAStageBytes;
    static constexpr uint32_t kTmemCols = 2 * MT < 32 ? 32 : 2 * MT;  // power of two >= 32
};

template <int MT>
constexpr size_t gemm_swap_smem_bytes(int stages) {
    return 1024 + (size_t)stages * SwapTraits<MT>::kStageBytes + sizeof(SmemCtl);
}

// Narrow form: [align slack][SmemCtl, 1 KiB multiple][stages x kbs B slots][stages x kbs A
// slots][room]. The UMMA of a B slot reads 128 rows (16 KiB) from the slot's start and that
// of an A slot MT rows, so the allocation extends 16 KiB - slot_b + MT x 128 - slot_a past the
// slots; the barriers lie before them, out of reach of those reads.
constexpr uint32_t kSwapCtlBytes = (sizeof(SmemCtl) + 1023) / 1024 * 1024;
template <int MT>
constexpr size_t gemm_swapn_smem_bytes(int stages, int kbs, uint32_t slot_b, uint32_t slot_a) {
    return 1024 + kSwapCtlBytes + (size_t)stages * kbs * (slot_b + slot_a) + (16384u - slot_b) +
           (SwapTraits<MT>::kAStageBytes - slot_a);
}

// MT accumulator columns of TMEM lane (row) `lane` of this warp's quarter -> D[m0 + j][n].
// The TMEM loads are warp-collective: every lane runs the loop, lanes with n >= N (or, in the
// narrow form, lanes past the CTA's rows of B: `valid` false) only skip their stores.
template <int MT, bool ACC16, bool EPI>
__device__ __forceinline__ void swap_epilogue_t(const GemmParams& p, uint32_t trow, int m0,
                                                int n, bool valid) {
    const int M = p.M;
    const bool in_n = valid && n < p.N;  // not warp-uniform: only the stores are skipped
    float badd = 0.f;
    if constexpr (EPI) badd = (p.bias != nullptr && in_n) ? __half2float(p.bias[n]) : 0.f;
    const float alpha = p.alpha;
    __half* col = p.D + n;
    const size_t ldd = (size_t)p.ldd;
    uint32_t r[16];
#pragma unroll 1
    for (int j0 = 0; j0 < MT && m0 + j0 < M; j0 += 16) {
        tmem_ld_32x32b_x16(trow + (uint32_t)j0, r);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
            const int m = m0 + j0 + jj;
            float v = ACC16 ? __half2float(__ushort_as_half((unsigned short)(r[jj] & 0xFFFFu)))
                            : __uint_as_float(r[jj]);
            if constexpr (EPI) {
                v = __fadd_rn(__fmul_rn(v, alpha), badd);  // two roundings, as the reference
                v = v > 0.f ? v : 0.f;
            }
            if (in_n && m < M) col[(size_t)m * ldd] = __float2half_rn(v);
        }
    }
}

// NARROW: the form for decode shapes whose 128-row blocks of B would leave most SMs idle.
// Each CTA takes p.swap_rb (< 128) rows of B -- ~N / SMs, so the whole B streams through
// every SM at once with no split-K and no cross-CTA reduction -- and a ring stage holds
// p.swap_kbs k-blocks (small boxes, enough bytes in flight). The UMMA is the same 128 x MT x
// 16: it reads 128 rows from the start of each B slot, the rows past swap_rb being whatever
// follows in shared memory; they only feed accumulator lanes >= swap_rb, which no epilogue
// lane stores. Per output element the k order is the 128-row form's, so results match it bit
// for bit.
template <int MT, bool NARROW = false>
__global__ void __launch_bounds__(kMaxThreads, 1)
    gemm_sm100_swap(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using ST = SwapTraits<MT>;
    clock_mark(0);
    extern __shared__ uint8_t smem_dyn[];
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    // k-block j of ring stage s lives in B slot and A slot s * kbs + j
    const int kbs = NARROW ? p.swap_kbs : 1;
    const int rb = NARROW ? p.swap_rb : 128;
    const uint32_t slot_b = NARROW ? p.swap_slot_b : ST::kBStageBytes;
    const uint32_t slot_a = NARROW ? p.swap_slot_a : ST::kAStageBytes;
    const uint32_t nslots = (uint32_t)(p.stages * kbs);
    const uint32_t sB = raw + pad + (NARROW ? kSwapCtlBytes : 0u);  // UMMA A operand: B rows
    const uint32_t sA = sB + nslots * slot_b;                     // UMMA B operand: A rows
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(
        smem_dyn + pad + (NARROW ? 0 : (size_t)nslots * (slot_b + slot_a)));

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
            mbar_init(tempty0 + 8 * b, 4);  // one arrive per epilogue warp (4 warps)
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
        tmem_alloc<1>(smem_u32(&ctl->tmem_base), ST::kTmemCols);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;
    volatile int* abort_flag = &ctl->abort;
    volatile int* no_abort = &ctl->never;
    grid_dep_wait();
    grid_dep_launch();

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
                const int m0 = tm * MT, n0 = tn * rb;
                for (int kb = 0; kb < p.num_kb; kb += kbs) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, w)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8 * stage;
                    // stage_tx: bytes of one k-block's two boxes
                    if (NARROW && p.swap_3d) {
                        // the whole stage in one box per operand (k-blocks past K zero-filled
                        // but counted: a box always lands whole)
                        const uint32_t slot = (uint32_t)(stage * kbs);
                        mbar_arrive_expect_tx(fb, (uint32_t)kbs * p.stage_tx);
                        tma_load_3d(sB + slot * slot_b, &tmB, fb, 0, n0, kb);
                        tma_load_3d(sA + slot * slot_a, &tmA, fb, 0, m0, kb);
                    } else {
                        // the last stage may be short
                        const int nk = NARROW ? min(kbs, p.num_kb - kb) : 1;
                        mbar_arrive_expect_tx(fb, (uint32_t)nk * p.stage_tx);
                        for (int j = 0; j < nk; ++j) {
                            const uint32_t slot = (uint32_t)(stage * kbs + j);
                            tma_load_2d(sB + slot * slot_b, &tmB, fb, (kb + j) * kBK, n0);
                            tma_load_2d(sA + slot * slot_a, &tmA, fb, (kb + j) * kBK, m0);
                        }
                    }
                    ++issued;
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
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
        // ------------------------------- MMA issuer -------------------------------
        const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitMma};
        const uint64_t adesc0 = sdesc_sw128(sB, 16, 1024);  // 128 rows of B
        const uint64_t bdesc0 = sdesc_sw128(sA, 16, 1024);  // MT rows of A
        const uint32_t idesc = p.idesc;
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1) & 1u;
            if (!mbar_wait_warp(tempty0 + 8 * buf, use ^ 1u, w)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(buf * MT);
            for (int kb = 0; kb < p.num_kb; kb += kbs) {
                if (!mbar_wait_warp(full0 + 8 * stage, phase, w)) {
                    ok = false;
                    break;
                }
                const int nk = NARROW ? min(kbs, p.num_kb - kb) : 1;
                if (elect_one()) {
                    for (int j = 0; j < nk; ++j) {
                        const uint32_t slot = (uint32_t)(stage * kbs + j);
                        const uint64_t ad = adesc0 + (uint64_t)((slot * slot_b) >> 4);
                        const uint64_t bd = bdesc0 + (uint64_t)((slot * slot_a) >> 4);
                        mma_f16_ss<1>(d_tmem, ad, bd, idesc, kb + j > 0 ? 1u : 0u);
                        mma_f16_ss<1>(d_tmem, ad + 2, bd + 2, idesc, 1u);
                        mma_f16_ss<1>(d_tmem, ad + 4, bd + 4, idesc, 1u);
                        mma_f16_ss<1>(d_tmem, ad + 6, bd + 6, idesc, 1u);
                    }
                    mma_commit(empty0 + 8 * stage);
                }
                __syncwarp();
                if (++stage == p.stages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if (elect_one()) mma_commit(tfull0 + 8 * buf);
            __syncwarp();
        }
        const WaitCtx wd{p.timeout_ns, no_abort, kErrWaitDrain};
        if (elect_one()) mma_commit(drain);
        __syncwarp();
        mbar_wait_warp(drain, 0, wd);
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------------
        const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitEpilogue};
        const int q = warp & 3;  // TMEM lane quarter = D columns n0 + 32q .. + 31
        const bool acc16 = p.acc_f16 != 0, epi = p.epilogue != 0;
        int it = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1) & 1u;
            const bool ok = mbar_wait(tfull0 + 8 * buf, use, w);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            int tm, tn;
            tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
            const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * MT);
            const int m0 = tm * MT, n = tn * rb + q * 32 + lane;
            // narrow form: quarters wholly past the CTA's rows of B have nothing to store
            if (!NARROW || q * 32 < rb) {
                const bool valid = !NARROW || q * 32 + lane < rb;
                if (acc16) {
                    if (epi)
                        swap_epilogue_t<MT, true, true>(p, trow, m0, n, valid);
                    else
                        swap_epilogue_t<MT, true, false>(p, trow, m0, n, valid);
                } else {
                    if (epi)
                        swap_epilogue_t<MT, false, true>(p, trow, m0, n, valid);
                    else
                        swap_epilogue_t<MT, false, false>(p, trow, m0, n, valid);
                }
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
        tmem_dealloc<1>(tmem_base, ST::kTmemCols);
    }
    clock_mark(1);
}

}  // namespace b2g
