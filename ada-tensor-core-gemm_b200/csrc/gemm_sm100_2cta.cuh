// gemm_sm100_2cta.cuh -- persistent FP16 GEMM on 2-CTA clusters (tcgen05 cta_group::2).
//
// A cluster of two CTAs on two SMs computes one 256 x BNP output tile (BNP = 128, 256 or
// 512) with UMMA 256 x N x 16 instructions issued by the even ("leader") CTA. Each CTA stages
// only its own half of the operands in shared memory -- 128 rows of A and BNP / 2 rows of B
// per k-block (32 KiB per stage at BNP = 256 instead of 48 KiB for a 128 x 256 tile on one
// SM) -- and the tensor core reads both CTAs' halves. Every CTA keeps its 128 rows of the
// accumulator in its own 512 TMEM columns. No TMA multicast is used: each CTA loads its
// halves itself (this code also runs on multi-GPU jobs).
//
// BNP = 128 and 256: the accumulator is double-buffered (two 256-column buffers), so the
// epilogue of one tile overlaps the mainloop of the next.
// BNP = 512 ("wide" pair tile): each CTA's 128 x 512 accumulator fills all 512 columns, as two
// 256-column halves issued as separate UMMA 256 x 256 x 16. Per k-block a CTA then loads
// 16 KiB of A and 32 KiB of B for twice the work, so the L2 -> SM traffic per FLOP drops by a
// quarter. There is no second accumulator; instead the halves are released separately: the
// epilogue drains half 0, frees it, then half 1, while the MMA warp starts the next tile on
// half 0 and defers the half-1 MMAs of up to 3 k-blocks (holding their stages) until half 1
// is free.
//
// Clusters: launched with a runtime cluster shape of 2 CTAs (one pair), or of 2 x S CTAs for
// split-K reduced through distributed shared memory (csplit): pair s of the cluster computes
// split s of the cluster's tile. Pair-local ranks: the CTA with cluster rank r is CTA r & 1 of
// its pair, whose leader has rank r & ~1.
//
// Work list: whole tiles first, then the tiles of the last, partial wave cut into
// `tail_split` (2 or 4) column slices (UMMA N = slice width <= 256; B read through a second
// tensor map whose box matches the slice), so the tail wave keeps every SM pair busy
// instead of leaving most of them idle. No workspace or reduction is needed.
//
// Roles (64 + 32 x 4 or 8 epilogue warps threads per CTA):
//   warp 0, one thread, both CTAs: TMA producer. Waits for its stage's `empty` barrier,
//     then loads its A half (128 x 64) and B half (width/2 x 64). Both CTAs' loads complete
//     on the LEADER's `full` barrier, which the leader's producer armed with the pair's
//     total byte count.
//   warp 1, leader only: MMA issuer (whole warp runs the loop, one elected lane issues).
//     Waits for `full` (both halves landed),
//     issues 4 x tcgen05.mma.cta_group::2, then a multicast tcgen05.commit that arrives on
//     the `empty` barrier of the same stage in both CTAs. After the last k-block, a
//     multicast commit on `tmem_full[buf]` of both CTAs.
//   warps 2.., both CTAs: epilogue of this CTA's 128 rows (same as the 1-CTA kernel),
//     then one arrive per warp on the leader's `tmem_empty[buf]` (count 2 x epilogue warps).
// Barrier waits are cluster-scope acquires (their arrivals come from the peer SM).
#pragma once

#include "gemm_sm100.cuh"

namespace b2g {

constexpr int kPairBM = 256;                       // pair tile rows (128 per CTA)
constexpr int kPairBN = 256;                       // UMMA N of one pair MMA
constexpr uint32_t kHalfBytes = 128 * kBK * 2;     // one operand half per k-block: 16 KiB
constexpr uint32_t kPairTmemCols = 512;            // 2 x 256 columns: buffers or halves

// Per-CTA shared memory of one stage: A half (16 KiB) + this CTA's BNP / 2 rows of B.
template <int BNP>
struct PairTraits {
    static_assert(BNP == 128 || BNP == 256 || BNP == 512, "pair tile width 128, 256 or 512");
    static constexpr uint32_t kBStageBytes = (uint32_t)BNP / 2 * kBK * 2;  // 16 or 32 KiB
    static constexpr uint32_t kStageBytes = kHalfBytes + kBStageBytes;
    static constexpr bool kWide = BNP == 512;
};

template <int BNP>
constexpr size_t gemm2_smem_bytes(int stages, uint32_t epi) {
    return 1024 + (size_t)stages * PairTraits<BNP>::kStageBytes + epi + sizeof(SmemCtl);
}

// Four UMMA 256 x N x 16 of one k-block into `d_tmem` (K steps: +32 B for A, +bk for B).
__device__ __forceinline__ void mma_kblock_pair(uint32_t d_tmem, uint64_t ad, uint64_t bd,
                                                uint32_t bk, uint32_t idesc, uint32_t acc0) {
    mma_f16_ss<2>(d_tmem, ad, bd, idesc, acc0);
    mma_f16_ss<2>(d_tmem, ad + 2, bd + bk, idesc, 1u);
    mma_f16_ss<2>(d_tmem, ad + 4, bd + 2 * bk, idesc, 1u);
    mma_f16_ss<2>(d_tmem, ad + 6, bd + 3 * bk, idesc, 1u);
}

// Work unit u -> tile index t, output tile (tm, tn), first output column and width of the
// unit, whether it is a tail slice, and its split-K index (split-K and tail slices are never
// combined: with splits > 1, unit u is split u % splits of tile u / splits).
template <int BNP, bool PLAIN = false>
__device__ __forceinline__ void pair_unit(const GemmParams& p, int u, int& t, int& tm, int& tn,
                                          int& n_first, int& width, bool& tail, int& split) {
    t = u;
    int sub = 0;
    split = 0;
    if (!PLAIN && p.splits > 1) {
        t = u / p.splits;
        split = u - t * p.splits;
        tail = false;
    } else {
        tail = u >= p.dp_tiles;
    }
    if (tail) {
        const int v = u - p.dp_tiles;
        t = p.dp_tiles + v / p.tail_split;
        sub = v - (t - p.dp_tiles) * p.tail_split;
    }
    tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
    width = tail ? BNP / p.tail_split : BNP;
    n_first = tn * BNP + sub * width;
}

// PEERS: the fused all-gather instantiation (every staged box of D also goes to p.peers).
// PLAIN: the instantiation for the common case -- no split-K, FP32 accumulation, plain store,
// B stored N x K, no peers -- with those modes as compile-time constants; CSPLIT: split-K
// reduced in a cluster, FP32 accumulation, no peers (see gemm_sm100_1cta).
template <int BNP, bool PEERS = false, bool PLAIN = false, bool CSPLIT = false>
__global__ void __launch_bounds__(kMaxThreads, 1)
    gemm_sm100_2cta(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmBt,
                    const __grid_constant__ CUtensorMap tmD, const GemmParams p) {
    static_assert(!(PEERS && (PLAIN || CSPLIT)) && !(PLAIN && CSPLIT), "one variant at a time");
    const int splits = PLAIN ? 1 : p.splits;
    const bool csplit = PLAIN ? false : CSPLIT ? true : p.csplit != 0;
    const bool b_mn = PLAIN ? false : p.b_mn_major != 0;
    const bool b_kn3d = PLAIN ? false : p.b_kn3d != 0;
    // k-blocks [kb0, kb1) of split s of a tile
    const auto krange = [&](int s, int& kb0, int& kb1) {
        if (PLAIN) {
            kb0 = 0;
            kb1 = p.num_kb;
        } else {
            split_range(p, s, kb0, kb1);
        }
    };
    clock_mark(0);
    B2G_TIC(t_life);
    if (threadIdx.x == 0) B2G_MARK(0);
    extern __shared__ uint8_t smem_dyn[];
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    using PT = PairTraits<BNP>;
    const uint32_t sA = raw + pad;
    const uint32_t sB = sA + (uint32_t)p.stages * kHalfBytes;
    const uint32_t sEpi = sA + (uint32_t)p.stages * PT::kStageBytes;
    const int epi_warps = (int)(blockDim.x >> 5) - 2;  // 4 or 8
    // cluster split-K receive slots: over the drained ring, or after the epilogue staging
    const uint32_t sRecv = p.recv_ring ? sA : sEpi + epi_bytes(epi_warps, p.epi_bufs);
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem_dyn + pad + (size_t)p.stages * PT::kStageBytes +
                                              epi_bytes(epi_warps, p.epi_bufs) +
                                              (p.recv_ring ? 0u : p.recv_bytes));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t crank = cluster_ctarank();
    const uint32_t rank = crank & 1u;               // this CTA's place in its pair
    const uint32_t lead = crank & ~1u;              // cluster rank of the pair's leader
    const uint16_t pair_mask = (uint16_t)(3u << lead);
    const bool leader = rank == 0;
    const int cluster_id = blockIdx.x >> 1, num_clusters = gridDim.x >> 1;
    const uint32_t full0 = smem_u32(&ctl->full[0]);
    const uint32_t empty0 = smem_u32(&ctl->empty[0]);
    const uint32_t tfull0 = smem_u32(&ctl->tmem_full[0]);
    const uint32_t tempty0 = smem_u32(&ctl->tmem_empty[0]);
    const uint32_t drain = smem_u32(&ctl->drain);
    const uint32_t rbar0 = smem_u32(&ctl->recv[0]);
    const uint32_t peers_free = smem_u32(&ctl->peers_free);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);   // only the leader's copy is used
            mbar_init(empty0 + 8 * s, 1);  // one multicast commit per use
        }
        if (csplit) {
            for (int k = 0; k < kCsMaxPieces; ++k) mbar_init(rbar0 + 8 * k, 1);  // owner's arm
            mbar_init(peers_free, p.recv_ring ? (uint32_t)(splits - 1) : 1u);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, 2u * epi_warps);  // epilogue warps x 2 CTAs (leader's copy)
        }
        mbar_init(drain, 1);
        ctl->abort = 0;
        ctl->never = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        prefetch_tmap(&tmBt);
        if (p.d_tma) prefetch_tmap(&tmD);
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
    const uint32_t full0_leader = mapa_shared(full0, lead);
    const uint32_t tempty0_leader = mapa_shared(tempty0, lead);
    // everything above overlapped the previous kernel; global memory only from here on
    if (threadIdx.x == 0) B2G_MARK(1);
    grid_dep_wait();
    grid_dep_launch();
    if (threadIdx.x == 0) B2G_MARK(2);

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------ TMA producer ------------------------------
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitProducer};
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = cluster_id; u < p.num_units && ok; u += num_clusters) {
                int t, tm, tn, n_first, width, split, kb0, kb1;
                bool tail;
                pair_unit<BNP, PLAIN>(p, u, t, tm, tn, n_first, width, tail, split);
                krange(split, kb0, kb1);
                const int m0 = tm * kPairBM + (int)rank * 128;
                // B of the unit in 256-column halves; this CTA loads hw rows of each
                const int nh = width > kPairBN ? 2 : 1;
                const int hw = (width > kPairBN ? kPairBN : width) >> 1;
                const CUtensorMap* mapB = tail ? &tmBt : &tmB;
                // pair total: 2 x (A half 16 KiB + B half width/2 rows x 128 B)
                const uint32_t bytes = 2u * (kHalfBytes + (uint32_t)(width >> 1) * 128u);
                if (u == cluster_id) B2G_MARK(10);
                for (int kb = kb0; kb < kb1; ++kb) {
                    B2G_TIC(t_empty);
                    if (!mbar_wait<true>(empty0 + 8 * stage, phase ^ 1u, w)) {
                        ok = false;
                        break;
                    }
                    B2G_TOC(0, t_empty);
                    if (kb == kb0 && u == cluster_id) B2G_MARK(11);
                    if (leader) mbar_arrive_expect_tx(full0 + 8 * stage, bytes);
                    const uint32_t fb = full0_leader + 8 * stage;
                    tma_load_2d_pair(sA + stage * kHalfBytes, &tmA, fb, kb * kBK, m0);
                    if (kb == kb0 && u == cluster_id) B2G_MARK(12);
                    for (int h = 0; h < nh; ++h) {
                        const int n0 = n_first + h * kPairBN + (int)rank * hw;
                        const uint32_t dst = sB + stage * PT::kBStageBytes + (uint32_t)h * kHalfBytes;
                        if (b_kn3d) {
                            // B is K x N: the hw / 64 boxes of 64 columns x 64 k-rows at once
                            tma_load_3d_pair(dst, mapB, fb, 0, kb * kBK, n0 >> 6);
                        } else if (b_mn) {
                            // B is K x N: hw / 64 boxes of 64 columns x 64 k-rows
                            for (int j = 0; j < (hw >> 6); ++j)
                                tma_load_2d_pair(dst + (uint32_t)j * kMnBoxBytes, mapB, fb,
                                                 n0 + 64 * j, kb * kBK);
                        } else {
                            tma_load_2d_pair(dst, mapB, fb, kb * kBK, n0);
                        }
                    }
                    if (kb == kb0 && u == cluster_id) B2G_MARK(3);
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
        if (leader) {
            // ------------------------------- MMA issuer -------------------------------
            // The whole warp runs the loop (operands stay warp-uniform); one elected lane
            // issues. Shared-memory descriptors are built once and advanced by adding the
            // stage offset (and 32 bytes per K step) to the start-address field: every
            // operand address is below 256 KiB, so the 14-bit field never carries.
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitMma};
            const uint64_t adesc0 = sdesc_sw128(sA, 16, 1024);
            const uint64_t bdesc0 = b_desc0(sB, b_mn);
            const uint32_t bk = b_kstep(b_mn);
            constexpr uint32_t kAStep = kHalfBytes >> 4;         // descriptor units per stage
            constexpr uint32_t kBStep = PT::kBStageBytes >> 4;
            constexpr uint32_t kBHalf = kHalfBytes >> 4;         // second 256-column half of B
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int u = cluster_id; u < p.num_units && ok; u += num_clusters, ++it) {
                int t, tm, tn, n_first, width, split, kb0, kb1;
                bool tail;
                pair_unit<BNP, PLAIN>(p, u, t, tm, tn, n_first, width, tail, split);
                krange(split, kb0, kb1);
                const uint32_t idesc = tail ? p.idesc_tail : p.idesc;
                const bool two_halves = PT::kWide && width > kPairBN;
                // 256-wide: double-buffered accumulators (buffer it & 1, reused every 2nd unit);
                // 512-wide: halves 0 / 1 of one accumulator, each freed once per unit
                const int buf = PT::kWide ? 0 : (it & 1);
                const uint32_t use = PT::kWide ? ((uint32_t)it & 1u) : ((uint32_t)(it >> 1) & 1u);
                B2G_TIC(t_te);
                if (!mbar_wait_warp<true>(tempty0 + 8 * buf, use ^ 1u, w)) {
                    ok = false;
                    break;
                }
                if (lane == 0) B2G_TOC(2, t_te);
                if (lane == 0) B2G_COUNT(7, 1);
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kPairBN);
                // 512-wide: the half-1 MMAs of the first k-blocks are deferred (their stages
                // held) while half 1 is still being drained by the previous unit's epilogue,
                // so the tensor pipe keeps working on half 0 meanwhile
                const int max_defer = two_halves ? (p.stages - 1 < 3 ? p.stages - 1 : 3) : 0;
                int deferred = 0, defer_stage = 0;
                bool half1_ready = !two_halves;
                // issue the deferred half-1 k-blocks (in k order) and free their stages
                auto flush_deferred = [&]() -> bool {
                    if (!mbar_wait_warp<true>(tempty0 + 8, use ^ 1u, w)) return false;
                    tc_fence_after();
                    half1_ready = true;
                    int st = defer_stage;
                    for (int i = 0; i < deferred; ++i) {
                        const uint64_t ad = adesc0 + (uint64_t)((uint32_t)st * kAStep);
                        const uint64_t bd = bdesc0 + (uint64_t)((uint32_t)st * kBStep);
                        if (elect_one()) {
                            mma_kblock_pair(d_tmem + (uint32_t)kPairBN, ad, bd + kBHalf, bk, idesc,
                                            i > 0 ? 1u : 0u);
                            mma_commit_pair(empty0 + 8 * st, pair_mask);
                        }
                        __syncwarp();
                        if (++st == p.stages) st = 0;
                    }
                    deferred = 0;
                    return true;
                };
                for (int kb = kb0; kb < kb1; ++kb) {
                    B2G_TIC(t_full);
                    if (!mbar_wait_warp(full0 + 8 * stage, phase, w)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) B2G_TOC(1, t_full);
                    if (lane == 0) B2G_COUNT(6, 1);
                    if (lane == 0 && kb == kb0 && it == 0) B2G_MARK(4);
                    const uint64_t ad = adesc0 + (uint64_t)((uint32_t)stage * kAStep);
                    const uint64_t bd = bdesc0 + (uint64_t)((uint32_t)stage * kBStep);
                    const uint32_t acc0 = kb > kb0 ? 1u : 0u;
                    if (elect_one()) mma_kblock_pair(d_tmem, ad, bd, bk, idesc, acc0);
                    __syncwarp();
                    bool commit = true;
                    if (two_halves) {
                        if (!half1_ready && deferred < max_defer) {
                            if (deferred == 0) defer_stage = stage;
                            ++deferred;
                            commit = false;  // held until its half-1 MMAs are issued
                        } else {
                            if (!half1_ready && !flush_deferred()) {
                                ok = false;
                                break;
                            }
                            if (elect_one())
                                mma_kblock_pair(d_tmem + (uint32_t)kPairBN, ad, bd + kBHalf, bk,
                                                idesc, acc0);
                            __syncwarp();
                        }
                    }
                    if (commit) {
                        if (elect_one()) mma_commit_pair(empty0 + 8 * stage, pair_mask);  // both CTAs
                        __syncwarp();
                    }
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                // a unit shorter than the deferral window ends with half-1 work pending
                if (ok && two_halves && !half1_ready && !flush_deferred()) ok = false;
                if (!ok) break;
                if (elect_one()) mma_commit_pair(tfull0 + 8 * buf, pair_mask);  // final in both CTAs
                __syncwarp();
                if (lane == 0) B2G_MARK(5);
            }
            const WaitCtx wd{p.timeout_ns, no_abort, kErrWaitDrain};
            if (elect_one()) mma_commit_2(drain);
            __syncwarp();
            mbar_wait_warp<true>(drain, 0, wd);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------------
        const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitEpilogue};
        const int q = warp & 3;
        const int c_first = (warp - 2) >> 2;
        const EpiScalars es = epi_scalars(p, epi_warps);
        const uint32_t stage0 = sEpi + (uint32_t)((warp - 2) * es.bufs) * kEpiBoxBytes;
        const bool acc16 = (PLAIN || CSPLIT) ? false : p.acc_f16 != 0;
        const bool epi = PLAIN ? false : p.epilogue != 0;
        uint32_t seq = 0;
        int it = 0;
        for (int u = cluster_id; u < p.num_units; u += num_clusters, ++it) {
            const int buf = PT::kWide ? 0 : (it & 1);
            const uint32_t use = PT::kWide ? ((uint32_t)it & 1u) : ((uint32_t)(it >> 1) & 1u);
            B2G_TIC(t_tf);
            const bool ok = mbar_wait<true>(tfull0 + 8 * buf, use, w);
            if (!__all_sync(0xffffffffu, ok)) break;
            if (warp == 2 && lane == 0) B2G_TOC(3, t_tf);
            if (warp == 2 && lane == 0) B2G_MARK(6);
            tc_fence_after();
            int t, tm, tn, n_first, width, split;
            bool tail;
            pair_unit<BNP, PLAIN>(p, u, t, tm, tn, n_first, width, tail, split);
            const int row0 = tm * kPairBM + (int)rank * 128 + q * 32;
            const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16);
            // accumulator buffer / half `b` has been read: the leader may reuse it
            auto release = [&](int b) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(tempty0_leader + 8 * b);
            };
            B2G_TIC(t_epi);
            if constexpr (PT::kWide) {
                // half 0 (columns [0, 256) of the unit), freed, then half 1; a unit of at most
                // 256 columns has an empty half 1, which is freed all the same so that both
                // halves complete one phase per unit
                for (int h = 0; h < 2; ++h) {
                    const int hw = width - h * kPairBN;
                    if (hw > 0)
                        epilogue_rows<PEERS>(p, es, &tmD, tq + (uint32_t)(h * kPairBN), row0,
                                             n_first + h * kPairBN, hw < kPairBN ? hw : kPairBN,
                                             c_first, stage0, lane, seq, acc16, epi);
                    release(h);
                }
            } else {
                const uint32_t tbase = tq + (uint32_t)(buf * kPairBN);
                if (splits > 1 && csplit) {
                    const int s = (int)(crank >> 1);
                    if (p.recv_ring && threadIdx.x == 64)
                        csplit_ring_free(peers_free, splits, s, 2, (int)rank);
                    csplit_epilogue<PEERS>(p, es, &tmD, tbase, q, BNP < kPairBN ? BNP : kPairBN,
                                           row0, n_first, c_first, stage0, lane, seq, epi, sRecv,
                                           rbar0, peers_free, w, [&] { release(buf); }, s, 2,
                                           (int)rank);
                } else if (splits > 1) {
                    splitk_epilogue<PEERS>(p, es, &tmD, tbase, t, split, (int)rank, 2, q,
                                           warp - 2, BNP < kPairBN ? BNP : kPairBN, row0, n_first,
                                           c_first, stage0, lane, seq, epi,
                                           [&] { release(buf); });
                } else {
                    epilogue_rows<PEERS>(p, es, &tmD, tbase, row0, n_first, width, c_first,
                                         stage0, lane, seq, acc16, epi);
                    release(buf);
                }
            }
            if (warp == 2 && lane == 0) B2G_TOC(4, t_epi);
            if (warp == 2 && lane == 0) B2G_MARK(7);
        }
        // this warp's TMA stores have read their staging boxes (their global writes complete
        // on their own; the kernel's completion makes them visible)
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        if (warp == 2 && lane == 0) B2G_MARK(8);
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
    if (threadIdx.x == 0) B2G_TOC(5, t_life);
    if (threadIdx.x == 0) B2G_MARK(9);
    clock_mark(1);
}

}  // namespace b2g
