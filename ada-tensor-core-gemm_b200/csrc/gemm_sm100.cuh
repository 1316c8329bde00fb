// gemm_sm100.cuh -- persistent, warp-specialised FP16 GEMM for sm_100a (one CTA per tile).
//
// Replaces the reference's gemm_kernel (src/gemm_bench.cu:213-399). The reference stages
// operands with per-thread cp.async into a STAGES-deep ring, moves them to registers with
// ldmatrix and multiplies with warp-level mma.sync, one CTA per output tile. Here:
//
//   warp 0 (1 thread)  TMA producer: for every k-block, wait for a free stage, then two
//                      cp.async.bulk.tensor loads (A 128x64, B BNx64, 128-byte swizzle)
//                      whose bytes complete the stage's `full` mbarrier.
//   warp 1             MMA issuer (the whole warp runs the loop, one elected lane issues):
//                      allocates TMEM (2 x BN columns: a double-buffered accumulator), waits
//                      for `full`, issues 4 tcgen05.mma (K = 16 each) reading both operands
//                      from shared memory, and tcgen05.commit's the stage's `empty` barrier;
//                      after the last k-block it commits `tmem_full[buf]`.
//   warps 2..          epilogue (4 or 8 warps): wait for `tmem_full[buf]`, tcgen05.ld 64
//                      columns at a time (warp w reads TMEM lanes 32*(w%4)..+31 = tile
//                      rows; with 8 warps two share a quarter, alternate chunks), apply the
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

// Most peer copies of D a fused all-gather writes (eight devices: seven peers).
constexpr int kMaxPeers = 7;
struct PeerCopies {
    int n;                     // copies in use (0: no fused all-gather)
    __half* d[kMaxPeers];      // D's first row in each copy
};

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
    int d_tma;       // D written by TMA stores (D 16-byte aligned and ldd % 8 == 0), else by
                     // coalesced plain stores from the same staging box
    int b_mn_major;  // B is K x N (MN-major) in global memory
    int b_kn3d;      // ... and read through a 3D tensor map (64 columns, K, N / 64): one load
                     // per CTA per stage brings all of its 64-column boxes (N % 64 == 0)
    unsigned long long timeout_ns;
    // 2-CTA kernel work list: tiles [0, dp_tiles) run whole; each remaining tile (the last,
    // partial wave) is cut into tail_split column slices of kPairBN / tail_split columns,
    // so the tail wave keeps every SM busy. num_units = dp_tiles + rest * tail_split.
    int dp_tiles, tail_split, num_units;
    uint32_t idesc_tail;
    // Split-K (FP32 accumulation only): unit u = tile (u / splits), k-blocks of split
    // (u % splits); see splitk_store / splitk_arrive_reduce. splits == 1: off.
    int splits;
    float* ws_part;                // FP32 partial accumulators, splitk_slot() layout
    unsigned long long* ws_count;  // arrival counters: (launch epoch << 32) | arrivals
    unsigned int epoch;            // this launch's epoch, never 0 and never repeated
    // splits > 1: csplit = 1 reduces the splits of a tile inside one cluster (`splits` CTAs,
    // or `splits` pairs of the 2-CTA kernel) through distributed shared memory (see
    // csplit_epilogue) instead of the workspace; the grid is then one CTA (pair) per unit,
    // not persistent. The receive slots (recv_bytes) either have their own shared memory after
    // the epilogue staging (recv_ring = 0: a split sends as soon as its own accumulator is
    // final) or overlay the drained operand ring (recv_ring = 1: more stages, but a split
    // sends only once every peer's ring has drained).
    int csplit;
    int recv_ring;
    uint32_t recv_bytes;
    // 1-CTA kernels: bytes one stage's two TMA loads deliver. When all of M fits one tile the
    // A box is only round_up(M, 8) rows high and the ring packs stages of a_stage_bytes of A
    // then B, so a decode-shaped GEMM fits several times more B stages in flight; the MMA still
    // reads 128 rows of A, the rows past the box coming from whatever follows in shared memory
    // (never past the allocation: the epilogue staging follows the ring), and they feed only
    // accumulator rows >= M, which the epilogue never stores.
    uint32_t stage_tx;
    uint32_t a_stage_bytes;  // A rows of one stage x 128 B (16 KiB for full 128-row tiles)
    // Epilogue staging: boxes of 4 KiB per epilogue warp (1..4), used in turn; the staging
    // area is epilogue warps x epi_bufs x 4 KiB, after the operand ring.
    int epi_bufs;
    // Fused all-gather: every staged box of D is also written, with 16-byte stores, to the
    // same rows and columns of npeer other copies of D (same ldd; peer devices' memory over
    // NVLink). The host guarantees N % 8 == 0, ldd % 8 == 0 and 16-byte aligned copies.
    PeerCopies peers;
    // Swapped-operand kernel, narrow form (decode shapes that give the 128-row form too few
    // CTAs): each CTA streams swap_rb (< 128) rows of B over the whole K range, swap_kbs
    // k-blocks per ring stage, each k-block's rows in a slot of swap_slot_b bytes (1 KiB
    // multiple). The UMMA still reads 128 rows: the rows past swap_rb come from whatever
    // follows in shared memory and feed only accumulator lanes the epilogue never stores.
    // swap_3d: K % 64 == 0 and rows in multiples of 8, so one 3D load per operand brings a
    // stage's swap_kbs k-blocks (box 64 x rows x k-blocks; slots of rows x 128 B, back to back).
    int swap_rb, swap_kbs, swap_3d;
    uint32_t swap_slot_b, swap_slot_a;
};

// k-blocks [kb0, kb1) of split s: an even share of the tile's num_kb k-blocks (32-bit
// arithmetic whenever splits x num_kb fits, as it does for any K below 2^22).
__device__ __forceinline__ void split_range(const GemmParams& p, int s, int& kb0, int& kb1) {
    if (p.num_kb <= 0xffff && p.splits <= 0xffff) {
        const uint32_t n = (uint32_t)p.num_kb, d = (uint32_t)p.splits;
        kb0 = (int)((uint32_t)s * n / d);
        kb1 = (int)((uint32_t)(s + 1) * n / d);
    } else {
        kb0 = (int)((long long)s * p.num_kb / p.splits);
        kb1 = (int)((long long)(s + 1) * p.num_kb / p.splits);
    }
}

constexpr int kBM = 128;      // rows of A per CTA (UMMA M for cta_group::1)
constexpr int kBK = 64;       // k-block: one 128-byte swizzle row of FP16
constexpr int kUmmaK = 16;    // K of one kind::f16 MMA
constexpr int kMaxStages = 8;
// Epilogue warps: 4 or 8, chosen at launch (blockDim.x = 64 + 32 x epilogue warps). Warp w
// may only read TMEM lanes 32*(w%4)..+31, so 4 warps cover the 128 accumulator rows once;
// with 8, two warps share each lane quarter and take alternate 64-column chunks. That halves
// the epilogue of a tile, which matters when K is small: the epilogue of tile i must finish
// within the (short) mainloop of tile i + 1, and D's write traffic dominates.
constexpr int kMaxEpiWarps = 8;
constexpr int kMaxThreads = 64 + 32 * kMaxEpiWarps;
__host__ __device__ constexpr int gemm_threads(int epi_warps) { return 64 + 32 * epi_warps; }
constexpr uint32_t kAStageBytes = kBM * kBK * 2;  // 16 KiB
// Epilogue staging for TMA stores: 32-row x 64-column FP16 boxes (4 KiB each, 128-byte
// swizzle), `epi_bufs` per epilogue warp, used in turn so the conversion of one chunk
// overlaps the bulk stores of the previous ones. Default 8 boxes in all (2 per warp with 4
// epilogue warps, 1 with 8); short-K launches trade ring stages for more boxes.
constexpr uint32_t kEpiBoxBytes = 32 * 64 * 2;
constexpr int kMaxEpiBufs = 4;
__host__ __device__ constexpr uint32_t epi_bytes(int epi_warps, int epi_bufs) {
    return (uint32_t)(epi_warps * epi_bufs) * kEpiBoxBytes;
}

// B operand layouts in shared memory (128-byte swizzle in both):
//   K-major (B stored N x K): rows of 64 k-values (128 B), 8-row atoms 1024 B apart (SBO);
//     a K step of 16 moves the start address by 32 B.
//   MN-major (B stored K x N): boxes of 64 n-values (128 B) x 64 k-rows, 8 KiB each and
//     placed back to back along N (LBO = 8 KiB between 64-column groups); 8 k-rows form a
//     1024 B atom (SBO); a K step of 16 moves the start address by 16 rows = 2 KiB.
constexpr uint32_t kMnBoxBytes = 64 * 64 * 2;
__device__ __forceinline__ uint64_t b_desc0(uint32_t sB, int b_mn_major) {
    return b_mn_major ? sdesc_sw128(sB, kMnBoxBytes, 1024) : sdesc_sw128(sB, 16, 1024);
}
// descriptor units (16 B) per UMMA K step of 16
__device__ __forceinline__ uint32_t b_kstep(int b_mn_major) { return b_mn_major ? 128u : 2u; }

template <int BN>
struct TileTraits {
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, step 64");
    static constexpr uint32_t kBStageBytes = BN * kBK * 2;
    static constexpr uint32_t kStageBytes = kAStageBytes + kBStageBytes;
    static constexpr uint32_t kTmemCols = 2 * BN;  // power of two for BN in {128, 256}
};

// Cluster split-K: most pieces (32 accumulator rows x 64 columns) one CTA owns and reduces,
// and the bytes of one FP32 piece.
constexpr int kCsMaxPieces = 8;
constexpr uint32_t kCsPieceBytes = 32 * 64 * 4;

struct SmemCtl {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t recv[kCsMaxPieces];  // cluster split-K: one receive barrier per owned piece
    uint64_t peers_free;          // cluster split-K: one arrival per peer whose ring drained
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    int never;  // stays 0: lets teardown waits ignore `abort` and use only their time limit
};

// Dynamic shared memory: [align slack][stages x (A, B)][epilogue staging][cluster split-K
// receive slots, unless they overlay the ring][SmemCtl]. A stage is a_rows x 128 B of A
// (a_rows = 128, or M rounded up to 8 when all of M fits one tile) followed by BN x 128 B of B.
template <int BN>
constexpr size_t gemm_smem_bytes(int stages, uint32_t epi, int a_rows = kBM) {
    return 1024 /* alignment slack */ +
           (size_t)stages * ((uint32_t)a_rows * kBK * 2 + TileTraits<BN>::kBStageBytes) + epi +
           sizeof(SmemCtl);
}

// The epilogue's per-element work uses only these scalars, read once from the kernel
// parameters into registers (per-element reads of GemmParams fields through a reference
// cost ~4x in the conversion loop).
struct EpiScalars {
    int M, N;
    float alpha;
    const __half* bias;
    int d_tma;
    uint64_t store_pol;  // L2 policy of the TMA stores of D: evict_first (D is not re-read)
    int bufs;            // staging boxes of this warp (1..4)
    int c_step;          // 64-column chunk stride of this warp (1 with 4 warps, 2 with 8)
};

__device__ __forceinline__ EpiScalars epi_scalars(const GemmParams& p, int epi_warps) {
    return EpiScalars{p.M, p.N, p.alpha, p.bias, p.d_tma, l2_policy_evict_first(), p.epi_bufs,
                      epi_warps / 4};
}

// alpha * acc + bias + ReLU (EPI) and round to FP16, two columns per word; ACC16: the
// accumulator is F16 in the low half of each 32-bit TMEM column.
template <bool ACC16, bool EPI>
__device__ __forceinline__ uint32_t epi_pack2(const EpiScalars& e, int col, uint32_t r0,
                                              uint32_t r1) {
    float v0, v1;
    if constexpr (ACC16) {
        v0 = __half2float(__ushort_as_half((unsigned short)(r0 & 0xFFFFu)));
        v1 = __half2float(__ushort_as_half((unsigned short)(r1 & 0xFFFFu)));
    } else {
        v0 = __uint_as_float(r0);
        v1 = __uint_as_float(r1);
    }
    if constexpr (EPI) {
        // multiply, then add: two roundings, as the reference's fused kernel computes them
        // (src/gemm_bench.cu:380-383; checked bit for bit against it on exact accumulators)
        v0 = __fmul_rn(v0, e.alpha);
        v1 = __fmul_rn(v1, e.alpha);
        if (e.bias != nullptr) {
            const int n0 = col < e.N ? col : e.N - 1;
            const int n1 = col + 1 < e.N ? col + 1 : e.N - 1;
            v0 = __fadd_rn(v0, __half2float(e.bias[n0]));
            v1 = __fadd_rn(v1, __half2float(e.bias[n1]));
        }
        v0 = v0 > 0.f ? v0 : 0.f;
        v1 = v1 > 0.f ? v1 : 0.f;
    }
    __half2 t = __floats2half2_rn(v0, v1);
    return *reinterpret_cast<uint32_t*>(&t);
}

// Staging box of this warp for its next TMA store: waits (lane 0) until the store that last
// read the box has finished reading it.
__device__ __forceinline__ uint32_t epi_box_acquire(const EpiScalars& e, uint32_t stage0,
                                                    uint32_t seq, int lane) {
    const uint32_t box = stage0 + (seq % (uint32_t)e.bufs) * kEpiBoxBytes;
    if (lane == 0) {  // at most bufs - 1 of this warp's stores may still be reading smem
        switch (e.bufs) {
            case 1: bulk_wait_read<0>(); break;
            case 2: bulk_wait_read<1>(); break;
            case 3: bulk_wait_read<2>(); break;
            default: bulk_wait_read<3>(); break;
        }
    }
    __syncwarp();
    return box;
}

// Convert 32 accumulator columns [col + 32h, col + 32h + 32) of row `lane` and write them as
// 16-byte groups j = 4h .. 4h + 3 of the box row (128-byte swizzle: group j of row r lives at
// (j ^ (r & 7)) * 16).
template <bool ACC16, bool EPI>
__device__ __forceinline__ void epi_box_put32(const EpiScalars& e, uint32_t box, int col, int h,
                                              const uint32_t (&r)[32], int lane) {
    const uint32_t rowaddr = box + (uint32_t)lane * 128u;
    const uint32_t sw = (uint32_t)(lane & 7);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const int j = 4 * h + jj, b = jj * 8, cc = col + j * 8;
        st_shared_v4(rowaddr + (((uint32_t)j ^ sw) << 4), epi_pack2<ACC16, EPI>(e, cc, r[b], r[b + 1]),
                     epi_pack2<ACC16, EPI>(e, cc + 2, r[b + 2], r[b + 3]),
                     epi_pack2<ACC16, EPI>(e, cc + 4, r[b + 4], r[b + 5]),
                     epi_pack2<ACC16, EPI>(e, cc + 6, r[b + 6], r[b + 7]));
    }
}

// Issue the TMA store of a filled box (lane 0); the tensor map clips the M / N edges.
__device__ __forceinline__ void epi_box_store(const EpiScalars& e, const CUtensorMap* tmD,
                                              uint32_t box, int col, int row0, int lane,
                                              uint32_t& seq) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d_hint(tmD, box, col, row0, e.store_pol);
        bulk_commit();
    }
    ++seq;
}

// Write a filled staging box to D with plain stores, for D that TMA cannot address (base
// not 16-byte aligned, or ldd not a multiple of 8): row by row, the lanes taking consecutive
// columns, so every store instruction covers 64 contiguous bytes of one row.
__device__ __forceinline__ void epi_box_store_rows(const GemmParams& p, const EpiScalars& e,
                                                   uint32_t box, int col, int row0, int lane) {
    __syncwarp();  // every lane's part of the box is written
    __half* const D = p.D;
    const long long ldd = p.ldd;
#pragma unroll 1
    for (int r = 0; r < 32 && row0 + r < e.M; ++r) {
        __half* drow = D + (size_t)(row0 + r) * (size_t)ldd;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int c = hh * 32 + lane;  // column within the box
            if (col + c < e.N) {
                const uint32_t off = (uint32_t)r * 128u +
                                     ((((uint32_t)c >> 3) ^ (uint32_t)(r & 7)) << 4) +
                                     ((uint32_t)c & 7u) * 2u;
                drow[col + c] = __ushort_as_half(ld_shared_u16(box + off));
            }
        }
    }
    __syncwarp();  // the box may be refilled
}

// Fused all-gather: copy a filled staging box (32 rows x 64 columns, 128-byte swizzle) to the
// same rows and columns of each peer copy of D. Lane l reads 16-byte group (l & 7) of rows
// (l >> 3) + 4i, i = 0..7, so each store instruction of the warp writes four whole 128-byte
// row segments. N % 8 == 0, so a group lies wholly inside or outside D. The stores are
// posted (nothing waits for them here); kernel completion makes them visible. Only the
// PEERS instantiations of the kernels contain this code.
template <bool PEERS>
__device__ __forceinline__ void epi_box_push(const GemmParams& p, const EpiScalars& e,
                                             uint32_t box, int col, int row0, int lane) {
    if constexpr (PEERS) {
        const int npeer = p.peers.n;
        __syncwarp();  // every lane's part of the box is written
        const int j = lane & 7, rq = lane >> 3;
        const int cg = col + j * 8;
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = rq + 4 * i;
            v[i] = ld_shared_v4(box + (uint32_t)r * 128u +
                                (((uint32_t)j ^ (uint32_t)(r & 7)) << 4));
        }
        const size_t ldd = (size_t)p.ldd;
        const size_t off = (size_t)(row0 + rq) * ldd + (size_t)cg;
        const int rows_left = e.M - row0 - rq;  // rows rq + 4i, 4i < rows_left, are inside D
        if (cg < e.N) {
#pragma unroll
            for (int q = 0; q < kMaxPeers; ++q) {  // constant indices into the parameters
                if (q < npeer) {
                    __half* dst = p.peers.d[q] + off;
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (4 * i < rows_left) st_global_cs_v4(dst + (size_t)(4 * i) * ldd, v[i]);
                }
            }
        }
        __syncwarp();  // the box may be refilled
    }
}

// Chunks c_first, c_first + e.c_step, ... (< nchunks) of 64 columns of this warp's 32 rows:
// TMEM -> registers 32 columns at a time -> convert -> swizzled staging box -> TMA store
// (d_tma), or coalesced plain stores of the box's rows. With two or more boxes per warp the
// chunks go in pairs: both boxes filled, then one generic->async proxy fence for the pair and
// two TMA stores (the per-chunk fence showed up as the epilogue's top "membar" stall; pairing
// measured +1.3% at 2048^3, +3% at 16384^2 x 256).
template <bool ACC16, bool EPI, bool PEERS>
__device__ __forceinline__ void epilogue_rows_t(const GemmParams& p, const EpiScalars& e,
                                                const CUtensorMap* tmD, uint32_t trow, int row0,
                                                int n_first, int nchunks, int c_first,
                                                uint32_t stage0, int lane, uint32_t& seq) {
    uint32_t r[32];
    if (e.d_tma && e.bufs >= 2) {
#pragma unroll 1
        for (int c = c_first; c < nchunks; c += 2 * e.c_step) {
            const int cn = c + e.c_step < nchunks ? 2 : 1;
            B2G_TIC(t_box);
            if (lane == 0) bulk_wait_read<0>();  // the previous pair's stores have read smem
            __syncwarp();
            B2G_TOC64(10, t_box);
            B2G_COUNT(12, threadIdx.x == 64 ? cn : 0);
            for (int i = 0; i < cn; ++i) {
                const int cc = c + i * e.c_step;
                const uint32_t box = stage0 + (uint32_t)i * kEpiBoxBytes;
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    tmem_ld_32x32b_x32(trow + (uint32_t)(cc * 64 + h * 32), r);
                    tmem_ld_wait();
                    if (threadIdx.x == 64 && c == c_first && i == 0 && h == 0) B2G_MARK(16);
                    epi_box_put32<ACC16, EPI>(e, box, n_first + cc * 64, h, r, lane);
                    if (threadIdx.x == 64 && c == c_first && i == 0 && h == 0) B2G_MARK(17);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                for (int i = 0; i < cn; ++i)
                    tma_store_2d_hint(tmD, stage0 + (uint32_t)i * kEpiBoxBytes,
                                      n_first + (c + i * e.c_step) * 64, row0, e.store_pol);
                bulk_commit();
            }
            if (threadIdx.x == 64 && c == c_first) B2G_MARK(18);
            for (int i = 0; i < cn; ++i)  // the TMA stores and these read the boxes together
                epi_box_push<PEERS>(p, e, stage0 + (uint32_t)i * kEpiBoxBytes,
                                    n_first + (c + i * e.c_step) * 64, row0, lane);
            seq += (uint32_t)cn;
        }
        return;
    }
#pragma unroll 1
    for (int c = c_first; c < nchunks; c += e.c_step) {
        const int col = n_first + c * 64;
        B2G_TIC(t_box);
        const uint32_t box = e.d_tma ? epi_box_acquire(e, stage0, seq, lane) : stage0;
        B2G_TOC64(10, t_box);
        B2G_COUNT(12, threadIdx.x == 64 ? 1 : 0);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
            tmem_ld_32x32b_x32(trow + (uint32_t)(c * 64 + h * 32), r);
            tmem_ld_wait();
            if (threadIdx.x == 64 && c == c_first && h == 0) B2G_MARK(16);
            epi_box_put32<ACC16, EPI>(e, box, col, h, r, lane);
            if (threadIdx.x == 64 && c == c_first && h == 0) B2G_MARK(17);
        }
        if (e.d_tma)
            epi_box_store(e, tmD, box, col, row0, lane, seq);
        else
            epi_box_store_rows(p, e, box, col, row0, lane);
        if (threadIdx.x == 64 && c == c_first) B2G_MARK(18);
        epi_box_push<PEERS>(p, e, box, col, row0, lane);
    }
}

// Epilogue of one warp: its 32 rows [row0, row0 + 32) x columns [n_first, n_first + width)
// (width <= 256) of the accumulator at TMEM address `trow` (lane quarter and buffer
// applied), 64 columns at a time: chunks c_first, c_first + e.c_step, ... (with 8 epilogue
// warps the other warp of the lane quarter takes the rest). `seq` counts this warp's issued
// TMA stores.
template <bool PEERS>
__device__ __forceinline__ void epilogue_rows(const GemmParams& p, const EpiScalars& e,
                                              const CUtensorMap* tmD, uint32_t trow, int row0,
                                              int n_first, int width, int c_first,
                                              uint32_t stage0, int lane, uint32_t& seq,
                                              bool acc16, bool epi) {
    if (row0 >= e.M) return;  // all 32 rows outside D (uniform in the warp)
    int nchunks = (width + 63) / 64;
    const int in_n = (e.N - n_first + 63) / 64;  // chunks that start inside D
    if (in_n < nchunks) nchunks = in_n;
    if (nchunks <= c_first) return;
    if (acc16) {
        if (epi)
            epilogue_rows_t<true, true, PEERS>(p, e, tmD, trow, row0, n_first, nchunks, c_first, stage0,
                                        lane, seq);
        else
            epilogue_rows_t<true, false, PEERS>(p, e, tmD, trow, row0, n_first, nchunks, c_first, stage0,
                                         lane, seq);
    } else {
        if (epi)
            epilogue_rows_t<false, true, PEERS>(p, e, tmD, trow, row0, n_first, nchunks, c_first, stage0,
                                         lane, seq);
        else
            epilogue_rows_t<false, false, PEERS>(p, e, tmD, trow, row0, n_first, nchunks, c_first,
                                          stage0, lane, seq);
    }
}

// ------------------------------------------------------------------------------------------
// Split-K. Each split of a tile writes its FP32 partial accumulator to the workspace and then
// counts itself in; the split that arrives last sums all partials in split order 0..S-1 (so
// the result does not depend on which split finished last) and runs the normal epilogue.
// Nothing ever waits for another CTA. Bookkeeping is per epilogue warp: warp w of every split
// covers the same 32 rows and 64-column chunks, so warp w of the last split needs only the
// partials of the other splits' warp w, and one counter per (tile, CTA of the pair, warp).
// ------------------------------------------------------------------------------------------

// Partial slot of (tile t, split s, CTA `rank`, lane quarter q): 32 rows x bn FP32, stored
// [64-column chunk][float4 index 0..15][lane] so every warp-wide store / load is one
// contiguous 512-byte run.
__device__ __forceinline__ float4* splitk_slot(const GemmParams& p, int t, int s, int rank,
                                               int ctas, int q, int bn) {
    const size_t slot = (((size_t)t * p.splits + s) * ctas + rank) * 4 + q;
    return reinterpret_cast<float4*>(p.ws_part + slot * 32 * (size_t)bn);
}

// Chunks [c_first, nchunks) step c_step of this warp's 32 rows, TMEM -> workspace partial.
__device__ __forceinline__ void splitk_store(float4* slot, uint32_t trow, int nchunks,
                                             int c_first, int c_step, int lane) {
    uint32_t r[32];
#pragma unroll 1
    for (int c = c_first; c < nchunks; c += c_step) {
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
            tmem_ld_32x32b_x32(trow + (uint32_t)(c * 64 + h * 32), r);
            tmem_ld_wait();
            float4* dst = slot + (size_t)c * 16 * 32 + h * 8 * 32 + lane;
#pragma unroll
            for (int v = 0; v < 8; ++v)
                dst[v * 32] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                          __uint_as_float(r[4 * v + 2]),
                                          __uint_as_float(r[4 * v + 3]));
        }
    }
}

// Count this warp's split of its tile in; true in every lane if it was the last of the
// `splits`. The counter holds (epoch << 32) | arrivals: the first arrival of a launch finds
// an older epoch (or 0) and starts over at 1, so no counter has to be cleared between
// launches, even after a launch that gave up half-way. Ordering: __syncwarp orders the
// lanes' partial stores before lane 0's release CAS (cumulative at gpu scope); the last
// arrival's CAS also acquires, and the lanes then read the other splits' partials from L2.
__device__ __forceinline__ bool splitk_arrive(unsigned long long* cnt, unsigned int epoch,
                                              int splits, int lane) {
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        const unsigned long long tag = (unsigned long long)epoch << 32;
        unsigned long long old = ld_relaxed_gpu_u64(cnt);
        bool done = false;
        for (int tries = 0; tries < (1 << 20) && !done; ++tries) {
            const unsigned long long next = (old & ~0xffffffffull) == tag ? old + 1 : tag + 1;
            const unsigned long long seen = atom_cas_acq_rel_gpu_u64(cnt, old, next);
            if (seen == old) {
                done = true;
                last = (int)(next & 0xffffffffull) == splits;
            } else {
                old = seen;
            }
        }
        if (!done) raise_status(kErrSplitCounter);
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();  // the lanes' partial loads are ordered after lane 0's acquire
    return last != 0;
}

// Last split: sum the partials of every split in split order 0..S-1, 16 columns at a time
// (the loads of four splits in flight together), and hand the sums to the
// normal epilogue (alpha, bias, ReLU, FP16, TMA store of each 64-column chunk).
template <bool EPI, bool PEERS>
__device__ __forceinline__ void splitk_reduce_t(const GemmParams& p, const EpiScalars& e,
                                                const CUtensorMap* tmD, int t, int rank,
                                                int ctas, int q, int bn, int row0, int n_first,
                                                int nchunks, int c_first, uint32_t stage0,
                                                int lane, uint32_t& seq) {
    const size_t split_stride = (size_t)32 * ctas * bn;  // float4s between splits' slots
    const float4* slot0 = splitk_slot(p, t, 0, rank, ctas, q, bn) + lane;
#pragma unroll 1
    for (int c = c_first; c < nchunks; c += e.c_step) {
        const int col = n_first + c * 64;
        const uint32_t box = e.d_tma ? epi_box_acquire(e, stage0, seq, lane) : stage0;
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {
            const float4* src = slot0 + (size_t)c * 512 + h * 128;
            float acc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = 0.f;
            // up to four splits' 16 columns in flight at once, added in split order
#pragma unroll 1
            for (int s0 = 0; s0 < p.splits; s0 += 4) {
                // splits past the last re-read split S - 1 (an L2 hit) and are not added
                float4 x[4][4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const float4* sg = src + (size_t)min(s0 + g, p.splits - 1) * split_stride;
#pragma unroll
                    for (int v = 0; v < 4; ++v) x[g][v] = __ldcg(sg + v * 32);
                }
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    if (s0 + g < p.splits) {
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            acc[4 * v] += x[g][v].x;
                            acc[4 * v + 1] += x[g][v].y;
                            acc[4 * v + 2] += x[g][v].z;
                            acc[4 * v + 3] += x[g][v].w;
                        }
                    }
                }
            }
            uint32_t r[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(acc[j]);
            // 16-byte groups j = 2h, 2h + 1 of row `lane` of the swizzled staging box
            const uint32_t rowaddr = box + (uint32_t)lane * 128u;
            const uint32_t sw = (uint32_t)(lane & 7);
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int j = 2 * h + jj, b = jj * 8, cc = col + j * 8;
                st_shared_v4(rowaddr + (((uint32_t)j ^ sw) << 4),
                             epi_pack2<false, EPI>(e, cc, r[b], r[b + 1]),
                             epi_pack2<false, EPI>(e, cc + 2, r[b + 2], r[b + 3]),
                             epi_pack2<false, EPI>(e, cc + 4, r[b + 4], r[b + 5]),
                             epi_pack2<false, EPI>(e, cc + 6, r[b + 6], r[b + 7]));
            }
        }
        if (e.d_tma)
            epi_box_store(e, tmD, box, col, row0, lane, seq);
        else
            epi_box_store_rows(p, e, box, col, row0, lane);
        epi_box_push<PEERS>(p, e, box, col, row0, lane);
    }
}

// Split-K epilogue of one warp for one unit: partial out, TMEM released through `release`
// (called once the accumulator has been read), then the reduction if this split was last.
template <bool PEERS, class Release>
__device__ __forceinline__ void splitk_epilogue(const GemmParams& p, const EpiScalars& e,
                                                const CUtensorMap* tmD, uint32_t trow, int t,
                                                int s, int rank, int ctas, int q, int wslot,
                                                int bn, int row0, int n_first, int c_first,
                                                uint32_t stage0, int lane, uint32_t& seq,
                                                bool epi, Release release) {
    // rows and chunks outside D are skipped identically by every split of the tile
    int nchunks = bn / 64;
    const int in_n = (e.N - n_first + 63) / 64;
    if (in_n < nchunks) nchunks = in_n;
    const bool active = row0 < e.M && nchunks > c_first;
    B2G_TIC(t_ps);
    if (active) splitk_store(splitk_slot(p, t, s, rank, ctas, q, bn), trow, nchunks, c_first,
                             e.c_step, lane);
    release();
    B2G_TOC64(13, t_ps);
    if (!active) return;
    unsigned long long* cnt = p.ws_count + ((size_t)t * ctas + rank) * kMaxEpiWarps + wslot;
    B2G_TIC(t_arr);
    const bool last = splitk_arrive(cnt, p.epoch, p.splits, lane);
    B2G_TOC64(14, t_arr);
    if (!last) return;
    B2G_TIC(t_red);
    B2G_COUNT(15, threadIdx.x == 64 ? 1 : 0);
    if (epi)
        splitk_reduce_t<true, PEERS>(p, e, tmD, t, rank, ctas, q, bn, row0, n_first, nchunks, c_first,
                              stage0, lane, seq);
    else
        splitk_reduce_t<false, PEERS>(p, e, tmD, t, rank, ctas, q, bn, row0, n_first, nchunks, c_first,
                               stage0, lane, seq);
    B2G_TOC64(12, t_red);
}

// ------------------------------------------------------------------------------------------
// Split-K reduced inside a cluster (1-CTA tiles, csplit). The grid has one CTA per unit and
// clusters of S = splits CTAs along x, so CTA rank s of a cluster computes split s of the
// cluster's tile; no workspace and no counters. The tile is cut into pieces of 32
// accumulator rows (one TMEM lane quarter q) x 64 columns (chunk c); piece i = q * chunks + c
// belongs to CTA i mod S of the cluster, as its (i / S)-th owned piece. The warp of every
// other split that holds the piece writes its FP32 values straight into the owner's shared
// memory with st.async, whose bytes complete the owner's receive barrier of that piece; the
// owner's warp sums the S partials in split order 0..S-1 (its own read from TMEM) -- the
// operations and order of the workspace reduction, so both give the same bits -- and runs the
// normal epilogue of the piece. Every receive slot is written once per launch, so no slot is
// ever reused and nothing waits for a free slot; senders never wait at all.
// ------------------------------------------------------------------------------------------

// Receive slots of one CTA: [owned piece k][sender slot j (senders in split order, the owner
// skipped)][float4 g 0..15][lane], so every warp-wide st.async / ld.shared is one contiguous
// 512-byte run.
__host__ __device__ constexpr uint32_t csplit_recv_bytes(int bn, int splits) {
    return (uint32_t)((4 * (bn / 64) + splits - 1) / splits) * (uint32_t)(splits - 1) *
           kCsPieceBytes;
}

// Send chunk c of this warp's 32 TMEM lanes to the owner: `dst` = the slot and `bar` = the
// owner's receive barrier, both as shared::cluster addresses.
__device__ __forceinline__ void csplit_send(uint32_t trow, int c, uint32_t dst, uint32_t bar,
                                            int lane) {
    uint32_t r[32];
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
        tmem_ld_32x32b_x32(trow + (uint32_t)(c * 64 + h * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < 8; ++g)
            st_async_v4(dst + (uint32_t)(((h * 8 + g) * 32 + lane) * 16), r[4 * g], r[4 * g + 1],
                        r[4 * g + 2], r[4 * g + 3], bar);
    }
}

// Owner: sum the S partials of chunk c in split order (own partial, split s, from TMEM; the
// others from the receive slots starting at `slots`) and store the piece like any epilogue.
template <bool EPI, bool PEERS>
__device__ __forceinline__ void csplit_reduce(const GemmParams& p, const EpiScalars& e,
                                              const CUtensorMap* tmD, uint32_t trow, int c,
                                              int s, uint32_t slots, int row0, int n_first,
                                              uint32_t stage0, int lane, uint32_t& seq) {
    const int S = p.splits;
    const int col = n_first + c * 64;
    const uint32_t box = e.d_tma ? epi_box_acquire(e, stage0, seq, lane) : stage0;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(trow + (uint32_t)(c * 64 + h * 32), r);
        tmem_ld_wait();
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.f;
#pragma unroll 1
        for (int t = 0; t < S; ++t) {
            if (t == s) {
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] += __uint_as_float(r[j]);
            } else {
                const uint32_t slot = slots + (uint32_t)(t < s ? t : t - 1) * kCsPieceBytes;
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const uint4 v = ld_shared_v4(slot + (uint32_t)(((h * 8 + g) * 32 + lane) * 16));
                    acc[4 * g] += __uint_as_float(v.x);
                    acc[4 * g + 1] += __uint_as_float(v.y);
                    acc[4 * g + 2] += __uint_as_float(v.z);
                    acc[4 * g + 3] += __uint_as_float(v.w);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(acc[j]);
        epi_box_put32<false, EPI>(e, box, col, h, r, lane);
    }
    if (e.d_tma)
        epi_box_store(e, tmD, box, col, row0, lane, seq);
    else
        epi_box_store_rows(p, e, box, col, row0, lane);
    epi_box_push<PEERS>(p, e, box, col, row0, lane);
}

// Cluster split-K: this CTA's ring has drained (its accumulator is final, so every load into
// the ring has landed and every MMA reading it is done): tell the CTAs that send to it -- the
// ones holding the same rows in the other splits -- that they may write its receive slots.
__device__ __forceinline__ void csplit_ring_free(uint32_t peers_free, int S, int s, int ctas,
                                                 int prank) {
    for (int o = 0; o < S; ++o)
        if (o != s) mbar_arrive_remote(mapa_shared(peers_free, (uint32_t)(o * ctas + prank)));
}

// Cluster split-K epilogue of one warp (lane quarter q, chunks c_first, c_first + c_step, ...)
// for this CTA's split s: first every piece another CTA owns is sent, then every owned piece
// is received (bounded wait) and reduced; TMEM is released last. Pieces outside D (rows >= M
// or chunks starting at or beyond N) are skipped by every split alike.
template <bool PEERS, class Release>
__device__ __forceinline__ void csplit_epilogue(const GemmParams& p, const EpiScalars& e,
                                                const CUtensorMap* tmD, uint32_t trow, int q,
                                                int bn, int row0, int n_first, int c_first,
                                                uint32_t stage0, int lane, uint32_t& seq,
                                                bool epi, uint32_t recv0, uint32_t rbar0,
                                                uint32_t peers_free, const WaitCtx& w,
                                                Release release, int s, int ctas, int prank) {
    // split s of the cluster; the CTA holding the same rows in split o has cluster rank
    // o * ctas + prank (ctas = 2 for the pair kernel, prank = this CTA's place in its pair)
    const int S = p.splits;
    const int nch = bn / 64;
    int nchunks = nch;
    const int in_n = (e.N - n_first + 63) / 64;
    if (in_n < nchunks) nchunks = in_n;
    if (threadIdx.x == 128) B2G_MARK(6);
    bool peers_ready = false;
    if (row0 < e.M) {
#pragma unroll 1
        for (int c = c_first; c < nchunks; c += e.c_step) {
            const int i = q * nch + c, owner = i % S, k = i / S;
            if (owner == s) continue;
            // slots over the owners' rings: send once every peer's ring has drained
            if (p.recv_ring && !peers_ready) {
                if (!mbar_wait_warp<true>(peers_free, 0, w)) break;
                peers_ready = true;
            }
            const int j = s < owner ? s : s - 1;
            const uint32_t orank = (uint32_t)(owner * ctas + prank);
            csplit_send(trow, c,
                        mapa_shared(recv0 + (uint32_t)(k * (S - 1) + j) * kCsPieceBytes, orank),
                        mapa_shared(rbar0 + 8u * (uint32_t)k, orank), lane);
        }
#pragma unroll 1
        for (int c = c_first; c < nchunks; c += e.c_step) {
            const int i = q * nch + c, owner = i % S, k = i / S;
            if (owner != s) continue;
            const uint32_t rb = rbar0 + 8u * (uint32_t)k;
            if (threadIdx.x == 128) B2G_MARK(7);
            if (lane == 0) mbar_arrive_expect_tx(rb, (uint32_t)(S - 1) * kCsPieceBytes);
            __syncwarp();
            B2G_TIC(t_rv);
            if (!mbar_wait_warp<true>(rb, 0, w)) break;
            B2G_TOC64(14, t_rv);
            if (threadIdx.x == 128) B2G_MARK(8);
            const uint32_t slots = recv0 + (uint32_t)(k * (S - 1)) * kCsPieceBytes;
            if (epi)
                csplit_reduce<true, PEERS>(p, e, tmD, trow, c, s, slots, row0, n_first, stage0,
                                           lane, seq);
            else
                csplit_reduce<false, PEERS>(p, e, tmD, trow, c, s, slots, row0, n_first, stage0,
                                            lane, seq);
        }
    }
    release();
    if (threadIdx.x == 128) B2G_MARK(9);
}

// PEERS: the fused all-gather instantiation (every staged box of D also goes to p.peers).
// PLAIN: the instantiation for the common case -- no split-K, FP32 accumulation, plain store,
// no peers -- in which those modes are compile-time constants, so the code a launch runs is
// only the plain path (fewer instruction-cache misses on its way, no integer divisions for
// split ranges); the host launches it whenever p allows. CSPLIT: likewise for split-K reduced
// in a cluster (FP32 accumulation, no peers), the decode-shaped launches.
template <int BN, bool PEERS = false, bool PLAIN = false, bool CSPLIT = false>
__global__ void __launch_bounds__(kMaxThreads, 1)
    gemm_sm100_1cta(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmD, const GemmParams p) {
    static_assert(!(PEERS && (PLAIN || CSPLIT)) && !(PLAIN && CSPLIT), "one variant at a time");
    using TT = TileTraits<BN>;
    const int splits = PLAIN ? 1 : p.splits;
    const bool csplit = PLAIN ? false : CSPLIT ? true : p.csplit != 0;
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
    // stage buffers must be 1024-byte aligned (128-byte swizzle atoms, base offset 0)
    const uint32_t raw = smem_u32(smem_dyn);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    // stage s: A at sA + s * stride, B at sB + s * stride
    const uint32_t stride = p.a_stage_bytes + TT::kBStageBytes;
    const uint32_t sA = raw + pad;
    const uint32_t sB = sA + p.a_stage_bytes;
    const uint32_t sEpi = raw + pad + (uint32_t)p.stages * stride;
    const int epi_warps = (int)(blockDim.x >> 5) - 2;  // 4 or 8
    // cluster split-K receive slots: over the drained ring, or after the epilogue staging
    const uint32_t sRecv = p.recv_ring ? sA : sEpi + epi_bytes(epi_warps, p.epi_bufs);
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem_dyn + pad + (size_t)p.stages * stride +
                                              epi_bytes(epi_warps, p.epi_bufs) +
                                              (p.recv_ring ? 0u : p.recv_bytes));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(&ctl->full[0]);
    const uint32_t empty0 = smem_u32(&ctl->empty[0]);
    const uint32_t tfull0 = smem_u32(&ctl->tmem_full[0]);
    const uint32_t tempty0 = smem_u32(&ctl->tmem_empty[0]);
    const uint32_t rbar0 = smem_u32(&ctl->recv[0]);
    const uint32_t peers_free = smem_u32(&ctl->peers_free);
    const uint32_t drain = smem_u32(&ctl->drain);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull0 + 8 * b, 1);
            mbar_init(tempty0 + 8 * b, (uint32_t)epi_warps);  // one arrive per epilogue warp
        }
        if (csplit) {
            for (int k = 0; k < kCsMaxPieces; ++k) mbar_init(rbar0 + 8 * k, 1);  // owner's arm
            mbar_init(peers_free, p.recv_ring ? (uint32_t)(splits - 1) : 1u);
        }
        mbar_init(drain, 1);
        ctl->abort = 0;
        ctl->never = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (p.d_tma) prefetch_tmap(&tmD);
    }
    if (warp == 1) {
        tmem_alloc<1>(smem_u32(&ctl->tmem_base), TT::kTmemCols);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    // cluster split-K: every CTA's receive barriers exist before any peer stores into them
    if (csplit) cluster_sync();
    tc_fence_after();
    if (threadIdx.x == 0) B2G_MARK(1);
    const uint32_t tmem_base = ctl->tmem_base;
    volatile int* abort_flag = &ctl->abort;
    volatile int* no_abort = &ctl->never;
    // the producer's first unit (tile and k-block range) is worked out while the previous
    // kernel may still be running, so its first load follows the wait directly
    int tm0 = 0, tn0 = 0, kb00 = 0, kb10 = 0;
    if (warp == 0 && lane == 0 && (int)blockIdx.x < p.num_units) {
        const int t = (int)blockIdx.x / splits;
        tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm0, tn0);
        krange((int)blockIdx.x - t * splits, kb00, kb10);
    }
    // everything above overlapped the previous kernel; global memory only from here on
    grid_dep_wait();
    grid_dep_launch();
    if (threadIdx.x == 0) B2G_MARK(2);

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------ TMA producer ------------------------------
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitProducer};
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
                int tm = tm0, tn = tn0, kb0 = kb00, kb1 = kb10;
                if (u != (int)blockIdx.x) {
                    const int t = u / splits;
                    tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
                    krange(u - t * splits, kb0, kb1);
                }
                const int m0 = tm * kBM, n0 = tn * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    B2G_TIC(t_empty);
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, w)) {
                        ok = false;
                        break;
                    }
                    B2G_TOC(0, t_empty);
                    if (issued == 0) B2G_MARK(15);
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_arrive_expect_tx(fb, p.stage_tx);
                    tma_load_2d(sA + stage * stride, &tmA, fb, kb * kBK, m0);
                    const uint32_t sBs = sB + stage * stride;
                    if (p.b_kn3d) {
                        // B is K x N: the BN / 64 boxes of 64 columns x 64 k-rows in one load
                        tma_load_3d(sBs, &tmB, fb, 0, kb * kBK, n0 >> 6);
                    } else if (p.b_mn_major) {
                        // B is K x N: BN / 64 boxes of 64 columns x 64 k-rows (8 KiB each)
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d(sBs + (uint32_t)j * kMnBoxBytes, &tmB, fb, n0 + 64 * j,
                                        kb * kBK);
                    } else {
                        tma_load_2d(sBs, &tmB, fb, kb * kBK, n0);
                    }
                    if (issued == 0) B2G_MARK(3);
                    ++issued;
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            B2G_MARK(11);
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
        {
            // ------------------------------- MMA issuer -------------------------------
            // Whole warp runs the loop (warp-uniform operands), one elected lane issues;
            // descriptors are advanced by adds (all operand addresses < 256 KiB).
            const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitMma};
            const uint64_t adesc0 = sdesc_sw128(sA, 16, 1024);
            const uint64_t bdesc0 = b_desc0(sB, p.b_mn_major);
            const uint32_t bk = b_kstep(p.b_mn_major);
            const uint32_t kAStep = stride >> 4, kBStep = stride >> 4;  // descriptor units
            const uint32_t idesc = p.idesc;
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x, ++it) {
                const int buf = it & 1;
                const uint32_t use = (uint32_t)(it >> 1) & 1u;
                int kb0, kb1;
                krange(u % splits, kb0, kb1);
                B2G_TIC(t_te);
                if (!mbar_wait_warp(tempty0 + 8 * buf, use ^ 1u, w)) {
                    ok = false;
                    break;
                }
                if (lane == 0) B2G_TOC(2, t_te);
                if (lane == 0) B2G_COUNT(7, 1);
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
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
                    if (elect_one()) {
                        mma_f16_ss<1>(d_tmem, ad, bd, idesc, kb > kb0 ? 1u : 0u);
                        mma_f16_ss<1>(d_tmem, ad + 2, bd + bk, idesc, 1u);
                        mma_f16_ss<1>(d_tmem, ad + 4, bd + 2 * bk, idesc, 1u);
                        mma_f16_ss<1>(d_tmem, ad + 6, bd + 3 * bk, idesc, 1u);
                        mma_commit(empty0 + 8 * stage);  // frees the stage once these retire
                    }
                    __syncwarp();
                    if (++stage == p.stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (elect_one()) mma_commit(tfull0 + 8 * buf);  // accumulator `buf` is final
                __syncwarp();
                if (lane == 0 && it == 0) B2G_MARK(5);
            }
            // drain: nothing may still read shared memory or write TMEM at teardown
            const WaitCtx wd{p.timeout_ns, no_abort, kErrWaitDrain};
            if (elect_one()) mma_commit(drain);
            __syncwarp();
            mbar_wait_warp(drain, 0, wd);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------------
        const WaitCtx w{p.timeout_ns, abort_flag, kErrWaitEpilogue};
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int c_first = (warp - 2) >> 2;  // first 64-column chunk of this warp
        const EpiScalars es = epi_scalars(p, epi_warps);
        const uint32_t stage0 = sEpi + (uint32_t)((warp - 2) * es.bufs) * kEpiBoxBytes;
        const bool acc16 = (PLAIN || CSPLIT) ? false : p.acc_f16 != 0;
        const bool epi = PLAIN ? false : p.epilogue != 0;
        uint32_t seq = 0;
        int it = 0;
        for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1) & 1u;
            B2G_TIC(t_tf);
            const bool ok = mbar_wait(tfull0 + 8 * buf, use, w);
            if (!__all_sync(0xffffffffu, ok)) break;
            if (warp == 2 && lane == 0) B2G_TOC(3, t_tf);
            B2G_TIC(t_epi);
            if (threadIdx.x == 64 && it == 0) B2G_MARK(12);
            tc_fence_after();
            const int t = u / splits;
            int tm, tn;
            tile_coord(t, p.tiles_m, p.tiles_n, p.group, tm, tn);
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
            auto release = [&] {  // accumulator `buf` has been read: the MMA warp may reuse it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
            };
            if (splits > 1 && csplit) {
                // tmem_full: every load of this CTA's ring has landed and every MMA reading it
                // is done, so the peers may overwrite the ring with their partials
                const int s = (int)cluster_ctarank();
                if (p.recv_ring && threadIdx.x == 64) csplit_ring_free(peers_free, splits, s, 1, 0);
                csplit_epilogue<PEERS>(p, es, &tmD, tbase, q, BN, tm * kBM + q * 32, tn * BN,
                                       c_first, stage0, lane, seq, epi, sRecv, rbar0, peers_free,
                                       w, release, s, 1, 0);
            } else if (splits > 1) {
                splitk_epilogue<PEERS>(p, es, &tmD, tbase, t, u - t * splits, 0, 1, q, warp - 2, BN,
                                tm * kBM + q * 32, tn * BN, c_first, stage0, lane, seq, epi,
                                release);
            } else {
                epilogue_rows<PEERS>(p, es, &tmD, tbase, tm * kBM + q * 32, tn * BN, BN, c_first,
                                     stage0, lane, seq, acc16, epi);
                release();
            }
            if (warp == 2 && lane == 0) B2G_TOC(4, t_epi);
            if (threadIdx.x == 64) B2G_MARK(13);
        }
        // this warp's TMA stores have read their staging boxes (their global writes complete
        // on their own; the kernel's completion makes them visible)
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        if (threadIdx.x == 64) B2G_MARK(14);
    }

    __syncthreads();
    // cluster split-K: no CTA leaves while a peer may still store into its receive slots
    if (csplit) cluster_sync();
    if (threadIdx.x == 0) B2G_MARK(10);
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, TT::kTmemCols);
    }
    if (threadIdx.x == 0) B2G_TOC(5, t_life);
    clock_mark(1);
}

}  // namespace b2g
