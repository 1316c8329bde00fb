// b2g_kernels.cu -- the device translation unit of libb200gemm.so: every sm_100a kernel of
// the library and the C-ABI entry points that launch them. (All device code lives in this
// one translation unit so the per-device status word g_b2g_status is a single symbol.)
//
// Launch boundary: b2g_gemm replaces the reference's run_cfg + pick dispatch
// (src/gemm_bench.cu:451-605): it validates the problem, builds the TMA tensor maps on the
// host, picks the tile configuration and launches the persistent kernel asynchronously.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "b2g.h"
#include "b2g_internal.h"
#include "aux_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_sm100_2cta.cuh"
#include "gemm_sm100_swap.cuh"
#include "probe_sm100.cuh"

namespace b2g {
namespace {

// ---------------------------------------------------------------------------------------
// TMA tensor maps
// ---------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// A 2-D FP16 tensor (outer x inner, inner contiguous, row pitch ld elements) read in boxes
// of box_outer x box_inner with 128-byte swizzle (box_inner * 2 must be 128).
int make_tmap(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
              uint32_t box_inner, uint32_t box_outer, const char* what) {
    auto enc = encode_fn();
    if (!enc) return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled(%s: %llu x %llu, ld %llu) failed: %d",
                    what, (unsigned long long)outer, (unsigned long long)inner,
                    (unsigned long long)ld, (int)r);
    return B2G_OK;
}

// B stored K x N as a 3D tensor: (64 columns, K rows, N / 64 column groups), strides ldb * 2
// bytes between rows and 128 bytes between groups, read in boxes of 64 columns x 64 k-rows x
// `groups` groups. TMA writes a box group after group, each group 64 rows of 128 bytes with
// 128-byte swizzle: exactly the MN-major operand layout of `groups` separate 2D boxes placed
// back to back, in one load. N must be a multiple of 64 so the groups tile N exactly (no load
// reads past the end of a row); groups past N / 64 read as zeros.
int make_tmap_kn3d(CUtensorMap* tm, const void* ptr, uint64_t N, uint64_t K, uint64_t ldb,
                   uint32_t groups) {
    auto enc = encode_fn();
    if (!enc) return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[3] = {64, K, N / 64};
    const cuuint64_t strides[2] = {ldb * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)kBK, groups};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled(B K x N in 3D, %llu x %llu, %u groups): %d",
                    (unsigned long long)K, (unsigned long long)N, groups, (int)r);
    return B2G_OK;
}

// One 3D load per stage for B stored K x N (default; B2G_KN3D=0 in the environment, read
// once per process, keeps the per-64-column 2D loads).
// 3D map over a row-major rows x K matrix (K % 64 == 0) whose box brings `kbs` consecutive
// k-blocks of `box_rows` rows in one load: dims (64, rows, K / 64), strides (ld x 2, 128 B);
// the k-blocks land back to back, box_rows x 128 B each. Rows past `rows` and k-blocks past
// K are zero-filled.
int make_tmap_kblocks(CUtensorMap* tm, const void* ptr, uint64_t rows, uint64_t K, uint64_t ld,
                      uint32_t box_rows, uint32_t kbs, const char* what) {
    auto enc = encode_fn();
    if (!enc) return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[3] = {64, rows, K / 64};
    const cuuint64_t strides[2] = {ld * 2, 128};
    const cuuint32_t box[3] = {64, box_rows, kbs};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(B2G_ERR_CUDA, "cuTensorMapEncodeTiled(%s in k-block boxes, %llu x %llu, box %u x %u): %d",
                    what, (unsigned long long)rows, (unsigned long long)K, box_rows, kbs, (int)r);
    return B2G_OK;
}

bool kn3d_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("B2G_KN3D");
        return !(e && e[0] == '0');
    }();
    return on;
}

// ---------------------------------------------------------------------------------------
// Per-device kernel set-up (opt-in shared memory), done once per kernel and device.
// ---------------------------------------------------------------------------------------
constexpr int kMaxDevices = 64;

// Geometry of the three GEMM kernels: output tile, CTAs per tile, TMA box rows per CTA.
struct TileGeom {
    int bm, bn;        // output tile of one CTA (1-CTA kernels) or of one CTA pair
    int ctas;          // CTAs per tile
    int box_a, box_b;  // rows of A / B that one CTA loads per k-block
};

TileGeom geom(int tile) {
    switch (tile) {
        case B2G_TILE_128x128: return {128, 128, 1, 128, 128};
        case B2G_TILE_128x256: return {128, 256, 1, 128, 256};
        case B2G_TILE_128x64: return {128, 64, 1, 128, 64};
        case B2G_TILE_256x512_2SM: return {kPairBM, 512, 2, 128, 128};
        case B2G_TILE_SWAP_AB: return {64, 128, 1, 64, 128};  // largest MT, for reports only
        case B2G_TILE_256x128_2SM: return {kPairBM, 128, 2, 128, 64};
        default: return {kPairBM, kPairBN, 2, 128, 128};
    }
}

// Instantiation of a GEMM kernel: the general one, the fused all-gather one (peers), the
// plain path (no split-K, FP32 accumulation, plain store, no peers; the pair kernel's also
// N x K B only) or split-K reduced in a cluster (FP32 accumulation, no peers); see
// gemm_sm100_1cta. The swapped-operand kernel has one instantiation.
enum KernelVariant { kVarGeneral = 0, kVarPeers = 1, kVarPlain = 2, kVarCsplit = 3, kVarNarrow = 4 };

#define B2G_VARIANTS_1CTA(BN)                                                        \
    (v == kVarPeers    ? (const void*)gemm_sm100_1cta<BN, true>                      \
     : v == kVarPlain  ? (const void*)gemm_sm100_1cta<BN, false, true>               \
     : v == kVarCsplit ? (const void*)gemm_sm100_1cta<BN, false, false, true>        \
                       : (const void*)gemm_sm100_1cta<BN>)
#define B2G_VARIANTS_2CTA(BNP)                                                       \
    (v == kVarPeers    ? (const void*)gemm_sm100_2cta<BNP, true>                     \
     : v == kVarPlain  ? (const void*)gemm_sm100_2cta<BNP, false, true>              \
     : v == kVarCsplit ? (const void*)gemm_sm100_2cta<BNP, false, false, true>       \
                       : (const void*)gemm_sm100_2cta<BNP>)

const void* kernel_ptr(int tile, int v = kVarGeneral) {
    switch (tile) {
        case B2G_TILE_128x128: return B2G_VARIANTS_1CTA(128);
        case B2G_TILE_128x256: return B2G_VARIANTS_1CTA(256);
        case B2G_TILE_128x64: return B2G_VARIANTS_1CTA(64);
        case B2G_TILE_256x512_2SM: return B2G_VARIANTS_2CTA(512);
        case B2G_TILE_SWAP_AB: return (const void*)gemm_sm100_swap<64>;
        case B2G_TILE_256x128_2SM: return B2G_VARIANTS_2CTA(128);
        default: return B2G_VARIANTS_2CTA(256);
    }
}
#undef B2G_VARIANTS_1CTA
#undef B2G_VARIANTS_2CTA

// Epilogue staging boxes (4 KiB each) of a launch, shared out among its epilogue warps: 16
// for K <= 256 (two per warp, so the 8 epilogue warps store chunks in fenced pairs: 16384^2 x
// 256 803 -> 827 TFLOP/s), else 8 (more boxes cost ring stages: -2% at K = 512, up to -15%
// at K >= 1024 with 24-32 boxes; stores in flight per warp are not the limit).
int epi_boxes_for(int num_kb) { return num_kb <= 4 ? 16 : 8; }

// `a_rows`: rows of A per stage of the 1-CTA kernels (128, or M rounded up to 8 when all of
// M fits one tile); the 2-CTA and swapped-operand kernels always stage full boxes.
size_t smem_needed(int tile, int stages, int epi_boxes = 8, int a_rows = kBM) {
    const uint32_t epi = (uint32_t)epi_boxes * kEpiBoxBytes;
    switch (tile) {
        case B2G_TILE_128x128: return gemm_smem_bytes<128>(stages, epi, a_rows);
        case B2G_TILE_128x256: return gemm_smem_bytes<256>(stages, epi, a_rows);
        case B2G_TILE_128x64: return gemm_smem_bytes<64>(stages, epi, a_rows);
        case B2G_TILE_256x512_2SM: return gemm2_smem_bytes<512>(stages, epi);
        case B2G_TILE_SWAP_AB: return gemm_swap_smem_bytes<64>(stages);
        case B2G_TILE_256x128_2SM: return gemm2_smem_bytes<128>(stages, epi);
        default: return gemm2_smem_bytes<256>(stages, epi);
    }
}

// Dynamic shared memory actually requested: at least just over half of the SM, so exactly
// one GEMM CTA is resident per SM. Every GEMM CTA allocates 2 x BN TMEM columns; two
// co-resident CTAs of 2-CTA clusters could otherwise each hold the TMEM the other's peer
// waits for.
size_t smem_request(int tile, int stages, const DeviceInfo& di, int epi_boxes = 8,
                    int a_rows = kBM) {
    return std::max(smem_needed(tile, stages, epi_boxes, a_rows),
                    (size_t)di.smem_per_sm / 2 + 1024);
}

int max_stages_for(int tile, int smem_optin, int epi_boxes = 8, int a_rows = kBM) {
    int s = kMaxStages;
    while (s > 2 && smem_needed(tile, s, epi_boxes, a_rows) > (size_t)smem_optin) --s;
    return s;
}

int ensure_kernel_attrs(int tile, const DeviceInfo& di, int v = kVarGeneral) {
    static bool done[4][7][kMaxDevices] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (di.device < kMaxDevices && done[v][tile][di.device]) return B2G_OK;
    cudaError_t e = cudaFuncSetAttribute(kernel_ptr(tile, v),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         di.smem_optin);
    if (e != cudaSuccess)
        return fail(B2G_ERR_CUDA, "cudaFuncSetAttribute(tile %d, max dynamic smem %d): %s", tile,
                    di.smem_optin, cudaGetErrorString(e));
    if (di.device < kMaxDevices) done[v][tile][di.device] = true;
    return B2G_OK;
}

// The instantiation a launch with these parameters takes (tile kernels with `ctas` CTAs per
// tile; the 1-CTA kernels' plain path reads B in either layout, the pair kernel's N x K only).
int kernel_variant(const GemmParams& p, int ctas) {
    if (p.peers.n > 0) return kVarPeers;
    if (p.splits == 1 && !p.csplit && !p.acc_f16 && !p.epilogue && (ctas == 1 || !p.b_mn_major))
        return kVarPlain;
    if (p.splits > 1 && p.csplit) return kVarCsplit;
    return kVarGeneral;
}

// Clusters of two that can be resident at once (GPCs with an odd SM count leave one idle).
int max_pair_clusters(const DeviceInfo& di, size_t smem) {
    static int cache[kMaxDevices] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (di.device < kMaxDevices && cache[di.device] > 0) return cache[di.device];
    ensure_kernel_attrs(B2G_TILE_256x256_2SM, di);  // the occupancy query needs its smem limit
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (di.sm_count / 2), 1, 1);
    cfg.blockDim = dim3(kMaxThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_sm100_2cta<256>, &cfg) != cudaSuccess ||
        n <= 0) {
        cudaGetLastError();
        n = di.sm_count / 2;
    }
    n = std::min(n, di.sm_count / 2);
    if (di.device < kMaxDevices) cache[di.device] = n;
    return n;
}

// Column-slice factor for the tail tiles of the 2-CTA kernel: the `rest` tiles of the last
// partial wave become rest * split units of 1/split the columns; pick the split (1, 2 or 4)
// that minimises the tail's duration ceil(rest * split / clusters) * cost(split). A slice
// costs more than 1/split of a tile because every slice reloads the tile's whole A panel
// (per k-block 16 KiB of A + 128 B x width/2 of B per CTA): measured on B200, a 128-column
// slice takes ~0.55 and a 64-column slice ~0.4 of a whole tile's time.
// For 256 x 512 tiles a 256-column slice is an ordinary 256 x 256 pair unit (~0.5 of the
// tile) and a 128-column slice ~0.3.
int tail_split_for(int rest, int clusters, int max_split, bool wide) {
    int best = 1;
    double best_t = 1.0;
    const double c2 = wide ? 0.50 : 0.55, c4 = wide ? 0.30 : 0.40;
    for (const auto& sc : {std::pair<int, double>{2, c2}, std::pair<int, double>{4, c4}}) {
        if (sc.first > max_split) continue;
        const double t = (double)((rest * sc.first + clusters - 1) / clusters) * sc.second;
        if (t < best_t - 1e-9) {
            best_t = t;
            best = sc.first;
        }
    }
    return best;
}

// L2 rasterization: the band of `group` M-tiles walked column-major keeps its A rows
// resident while B streams through. The band's A panel is sized to ~30% of the 126 MB L2
// (rounded, capped at the number of M-tiles): measured on B200 with 256 x 256 tiles, 8192^3
// runs best at 8 M-tiles (32 MiB of A; DRAM reads 1.09 GB vs 1.27 GB at 14), 16384^2 x 4096
// at 16, 16384^3 at 5-6; larger bands lose the streaming B panels from L2.
int auto_group(const TileGeom& g, int tiles_m, int K) {
    const double panel = (double)g.bm * (double)K * 2.0;  // bytes of A per M-tile
    int grp = (int)std::lround(0.30 * 126.0 * 1024 * 1024 / panel);
    grp = std::max(1, std::min(grp, tiles_m));
    return grp;
}

// Programmatic dependent launch (default on; B2G_PDL=0 turns it off): the GEMM's prologue
// overlaps the previous kernel in the stream, and its griddepcontrol.wait orders all of its
// global-memory accesses after that kernel. Every GEMM grid is fully co-resident
// (persistent, <= one CTA per SM), so a dependent grid can never hold SMs this one needs.
bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("B2G_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Epilogue warps of a launch: 8 when K <= 1024 (at most 16 k-blocks per tile: the next
// tile's mainloop is too short to hide a 4-warp epilogue, and D's writes dominate), else 4.
// B2G_EPI_WARPS=4 or 8 in the environment forces one (read once per process).
int epi_warps_for(int num_kb, int splits, bool wide, bool one_unit_per_cta) {
    static const int forced = [] {
        const char* e = std::getenv("B2G_EPI_WARPS");
        return e ? std::atoi(e) : 0;
    }();
    if (forced == 4 || forced == 8) return forced;
    // split-K: the reduction wants 8 as well; 256 x 512 tiles: the MMA warp waits for the
    // epilogue of half 1 at the start of every tile. A CTA with a single tile has no next
    // mainloop for its epilogue to keep up with: 4 (measured on B200, device time: 512^3
    // 5.05 -> 4.80 us, 1024^3 8.10 -> 7.81 us)
    if (splits > 1 || wide) return 8;
    if (one_unit_per_cta) return 4;
    return num_kb <= 16 ? 8 : 4;
}

// The most recent GEMM launch of this host thread (b2g_last_launch, b2g_last_launch_cluster).
struct LaunchRecord {
    int grid, threads, tile, stages, units, splits, cluster;
    int variant;  // KernelVariant of the tile kernels; the swapped-operand kernel: general
};
thread_local LaunchRecord g_last_launch = {};

// Launch with programmatic dependent launch (when enabled) and, for cluster > 1, a runtime
// cluster shape of `cluster` CTAs along x (kernels without __cluster_dims__).
template <class Kern, class... Args>
cudaError_t launch_exc(Kern kern, int grid, int threads, size_t smem, cudaStream_t s,
                       int cluster, const Args&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = (unsigned)na;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <class Kern, class... Args>
cudaError_t launch_ex(Kern kern, int grid, int threads, size_t smem, cudaStream_t s,
                      const Args&... args) {
    return launch_exc(kern, grid, threads, smem, s, 1, args...);
}

// Split-K reduced through distributed shared memory (csplit) unless B2G_SPLITK_CLUSTER=0 in
// the environment (read once per process), which keeps every split on the workspace path.
bool csplit_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("B2G_SPLITK_CLUSTER");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Whether clusters of `ctas` CTAs of the 1-CTA kernel `tile` (one per SM at this shared-
// memory size) can be resident on this device at all; cached per (device, tile, ctas, smem).
bool cluster_fits(const DeviceInfo& di, int tile, int ctas, int threads, size_t smem,
                  bool peers) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, size_t, bool>, bool> cache;
    const auto key = std::make_tuple(di.device, tile, ctas, smem, peers);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas, 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ctas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const bool ok = cudaOccupancyMaxActiveClusters(
                        &n, kernel_ptr(tile, peers ? kVarPeers : kVarCsplit), &cfg) ==
                        cudaSuccess &&
                    n > 0;
    if (!ok) cudaGetLastError();
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = ok;
    return ok;
}

// One launch of instantiation V (KernelVariant) of a tile kernel.
template <int V>
cudaError_t launch_gemm_t(int tile, const CUtensorMap& tmA, const CUtensorMap& tmB,
                          const CUtensorMap& tmBt, const CUtensorMap& tmD, const GemmParams& p,
                          const DeviceInfo& di, size_t smem, cudaStream_t s, int threads,
                          int& grid) {
    constexpr bool PEERS = V == kVarPeers, PLAIN = V == kVarPlain, CS = V == kVarCsplit;
    const int grid1 = p.csplit ? p.num_units : std::min(p.num_units, di.sm_count);
    const int cl1 = p.csplit ? p.splits : 1;
    const int grid2 =
        2 * (p.csplit ? p.num_units : std::min(p.num_units, max_pair_clusters(di, smem)));
    const int cl2 = p.csplit ? 2 * p.splits : 2;
    switch (tile) {
        case B2G_TILE_128x128:
            grid = grid1;
            return launch_exc(gemm_sm100_1cta<128, PEERS, PLAIN, CS>, grid, threads, smem, s, cl1,
                              tmA, tmB, tmD, p);
        case B2G_TILE_128x256:
            grid = grid1;
            return launch_exc(gemm_sm100_1cta<256, PEERS, PLAIN, CS>, grid, threads, smem, s, cl1,
                              tmA, tmB, tmD, p);
        case B2G_TILE_128x64:
            grid = grid1;
            return launch_exc(gemm_sm100_1cta<64, PEERS, PLAIN, CS>, grid, threads, smem, s, cl1,
                              tmA, tmB, tmD, p);
        case B2G_TILE_256x512_2SM:
            grid = grid2;
            return launch_exc(gemm_sm100_2cta<512, PEERS, PLAIN, CS>, grid, threads, smem, s, cl2,
                              tmA, tmB, tmBt, tmD, p);
        case B2G_TILE_256x128_2SM:
            grid = grid2;
            return launch_exc(gemm_sm100_2cta<128, PEERS, PLAIN, CS>, grid, threads, smem, s, cl2,
                              tmA, tmB, tmBt, tmD, p);
        default:
            grid = grid2;
            return launch_exc(gemm_sm100_2cta<256, PEERS, PLAIN, CS>, grid, threads, smem, s, cl2,
                              tmA, tmB, tmBt, tmD, p);
    }
}

int launch_gemm(int tile, const CUtensorMap& tmA, const CUtensorMap& tmB,
                const CUtensorMap& tmBt, const CUtensorMap& tmD, const GemmParams& p,
                const DeviceInfo& di, size_t smem, cudaStream_t s, int epi_warps) {
    const int v = kernel_variant(p, geom(tile).ctas);
    if (int rc = ensure_kernel_attrs(tile, di, v)) return rc;
    int grid = 0;
    const int threads = gemm_threads(epi_warps);
    cudaError_t e;
    switch (v) {
        case kVarPeers:
            e = launch_gemm_t<kVarPeers>(tile, tmA, tmB, tmBt, tmD, p, di, smem, s, threads, grid);
            break;
        case kVarPlain:
            e = launch_gemm_t<kVarPlain>(tile, tmA, tmB, tmBt, tmD, p, di, smem, s, threads, grid);
            break;
        case kVarCsplit:
            e = launch_gemm_t<kVarCsplit>(tile, tmA, tmB, tmBt, tmD, p, di, smem, s, threads, grid);
            break;
        default:
            e = launch_gemm_t<kVarGeneral>(tile, tmA, tmB, tmBt, tmD, p, di, smem, s, threads, grid);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(B2G_ERR_CUDA, "GEMM launch (tile %d, grid %d, smem %zu): %s", tile, grid, smem,
                    cudaGetErrorString(e));
    const int cluster = (p.csplit ? p.splits : 1) * geom(tile).ctas;
    g_last_launch = LaunchRecord{grid, threads, tile, p.stages, p.num_units, p.splits, cluster, v};
    return B2G_OK;
}

// ---------------------------------------------------------------------------------------
// Swapped-operand kernel for small M (tile B2G_TILE_SWAP_AB)
// ---------------------------------------------------------------------------------------
// MT (UMMA N = rows of A per CTA) so that the grid has about one CTA per SM: 128-column
// blocks of D times ceil(M / MT) row blocks.
int swap_mt_for(int M, int N, int sm_count) {
    const int n_tiles = (N + 127) / 128;
    const int target = std::max(1, sm_count / std::max(1, n_tiles));
    const int rows = (M + target - 1) / target;
    const int mt = rows <= 16 ? 16 : rows <= 32 ? 32 : 64;
    // launch_swap takes the narrow form when the 128-row blocks would leave more than half of
    // the SMs idle; it spreads N over the SMs itself, so it wants M in as few blocks as
    // possible (each M block re-reads all of B)
    if (2LL * ((M + mt - 1) / mt) * n_tiles < sm_count) return M <= 16 ? 16 : M <= 32 ? 32 : 64;
    return mt;
}

template <int MT>
int launch_swap(const void* A, const void* B, int M, int N, int K, long long lda, long long ldb,
                GemmParams& p, int stages, const DeviceInfo& di, cudaStream_t s) {
    using ST = SwapTraits<MT>;
    // The narrow form when 128-row blocks of B would leave more than half of the SMs idle:
    // ~N / (SMs per M-block) rows of B per CTA (8..64), so every SM streams its share of B
    // over the whole K range (measured on B200, N = K = 4096, device time, against the
    // 128-row form: M = 1 16.6 -> 12.0 us, M = 32 17.0 -> 13.4 us; the automatic choice there,
    // 128 x 128 tiles with cluster split-K, takes 11.6-11.7 us).
    const int tiles_m = (M + MT - 1) / MT;
    const bool narrow = 2LL * tiles_m * ((N + 127) / 128) < di.sm_count;
    int rb = 128, kbs = 1;
    uint32_t slot_b = ST::kBStageBytes, slot_a = ST::kAStageBytes;
    // A box rows: all of M in one block -> only round_up(M, 8) rows are loaded; the MMA reads
    // MT rows, the rows past the box feeding only D^T columns >= M, which are never stored
    int a_rows = MT;
    // K % 64 == 0: one 3D load per operand and stage, with rows in multiples of 8 so every
    // k-block's slot starts on a 1 KiB swizzle atom (else one 2D load per k-block and operand)
    const bool three_d = narrow && K % 64 == 0;
    if (narrow) {
        const int per_m = std::max(1, di.sm_count / tiles_m);
        const int step = three_d ? 8 : 4;
        rb = (N + per_m - 1) / per_m;
        rb = std::min(64, std::max(8, (rb + step - 1) / step * step));
        slot_b = (uint32_t)((rb * kBK * 2 + 1023) / 1024 * 1024);
        if (tiles_m == 1) a_rows = std::min(MT, (M + 7) / 8 * 8);
        if (three_d) slot_a = (uint32_t)a_rows * kBK * 2;
        // stages of ~32 KiB (a box's third dimension is at most 256 k-blocks)
        kbs = std::min(256, std::max(1, (int)(32768u / (slot_b + slot_a))));
    }
    const auto smem_for = [&](int st) {
        return narrow ? gemm_swapn_smem_bytes<MT>(st, kbs, slot_b, slot_a)
                      : gemm_swap_smem_bytes<MT>(st);
    };
    static bool done[2][kMaxDevices] = {};
    static std::mutex mu;
    const void* kern = narrow ? (const void*)gemm_sm100_swap<MT, true>
                              : (const void*)gemm_sm100_swap<MT, false>;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!(di.device < kMaxDevices && done[narrow][di.device])) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 di.smem_optin);
            if (e != cudaSuccess)
                return fail(B2G_ERR_CUDA, "cudaFuncSetAttribute(swap kernel): %s",
                            cudaGetErrorString(e));
            if (di.device < kMaxDevices) done[narrow][di.device] = true;
        }
    }
    if (stages == 0) {
        stages = kMaxStages;
        while (stages > 2 && smem_for(stages) > (size_t)di.smem_optin) --stages;
    }
    if (smem_for(stages) > (size_t)di.smem_optin)
        return fail(B2G_ERR_SMEM, "smem over per-block opt-in limit (swap kernel, %d stages)",
                    stages);
    const size_t smem = std::max(smem_for(stages), (size_t)di.smem_per_sm / 2 + 1024);
    p.stages = stages;
    p.tiles_m = tiles_m;
    p.tiles_n = (N + rb - 1) / rb;
    const long long nt = (long long)p.tiles_m * p.tiles_n;
    if (nt > 0x7fffffffLL) return fail(B2G_ERR_ARG, "too many tiles (%lld)", nt);
    p.num_tiles = p.num_units = p.dp_tiles = (int)nt;
    p.tail_split = 1;
    p.splits = 1;
    p.idesc = p.idesc_tail = idesc_f16(128, MT, p.acc_f16 == 0, false);
    // bytes one k-block's two boxes deliver
    p.stage_tx = (uint32_t)(rb + a_rows) * kBK * 2;
    p.swap_rb = rb;
    p.swap_kbs = kbs;
    p.swap_3d = three_d ? 1 : 0;
    p.swap_slot_b = slot_b;
    p.swap_slot_a = slot_a;
    if (p.group <= 0) p.group = 1;
    CUtensorMap tmA, tmB;
    if (three_d) {
        if (int rc = make_tmap_kblocks(&tmA, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda,
                                       (uint32_t)a_rows, (uint32_t)kbs, "A"))
            return rc;
        if (int rc = make_tmap_kblocks(&tmB, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb,
                                       (uint32_t)rb, (uint32_t)kbs, "B"))
            return rc;
    } else {
        if (int rc = make_tmap(&tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, kBK,
                               (uint32_t)a_rows, "A"))
            return rc;
        if (int rc = make_tmap(&tmB, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, kBK,
                               (uint32_t)rb, "B"))
            return rc;
    }
    const int grid = std::min(p.num_units, di.sm_count);
    const int threads = gemm_threads(4);
    cudaError_t e = narrow ? launch_ex(gemm_sm100_swap<MT, true>, grid, threads, smem, s, tmA,
                                       tmB, p)
                           : launch_ex(gemm_sm100_swap<MT, false>, grid, threads, smem, s, tmA,
                                       tmB, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(B2G_ERR_CUDA, "swap GEMM launch (MT %d, grid %d): %s", MT, grid,
                    cudaGetErrorString(e));
    g_last_launch = LaunchRecord{grid, threads, B2G_TILE_SWAP_AB, p.stages, p.num_units, 1, 1,
                                 narrow ? kVarNarrow : kVarGeneral};
    return B2G_OK;
}

// ---------------------------------------------------------------------------------------
// Split-K
// ---------------------------------------------------------------------------------------
// Automatic split factor. Only 1-CTA tiles are split, and only when the tiles fill less
// than half of the SMs: the S in 1..4 (one wave) minimising a cycle estimate of one unit,
//   ceil(num_kb / S) k-blocks x ~450 cycles + (S > 1) x ~10500 cycles,
// the second term being the split overhead measured on B200 for a 128 x 128 tile (partial
// store ~1.7K, arrival ~3K, the last split's reduction ~5.5K cycles, nearly independent of
// S <= 4). For 2-CTA pair tiles the overhead is ~3x larger and splitting measured slower on
// every shape tried, so pairs are never split automatically.
int splitk_auto(int tiles, int concurrent, int num_kb, int ctas) {
    if (ctas != 1 || 2 * tiles > concurrent) return 1;
    int best = 1;
    double best_t = num_kb * 450.0;
    for (int s = 2; s <= 4 && tiles * s <= concurrent; ++s) {
        const double t = ((num_kb + s - 1) / s) * 450.0 + 10500.0;
        if (t < best_t) {
            best_t = t;
            best = s;
        }
    }
    return best;
}

// Scratch of one split-K launch: FP32 partials, arrival counters and the launch's epoch.
struct SplitScratch {
    float* part;
    unsigned long long* count;
    unsigned int epoch;
};

// Library-owned split-K workspace, one per (device, stream) so GEMMs on different streams
// never share partials or counters; launches on one stream are ordered by the stream.
// It grows on demand (synchronising the stream first, since in-flight launches may still use
// the old buffers); growing is refused while the stream is being captured into a graph.
// Counters need no clearing between launches (epoch tags); a new counter buffer is zeroed.
struct StreamWorkspace {
    float* part = nullptr;
    size_t part_bytes = 0;
    unsigned long long* count = nullptr;
    size_t count_entries = 0;
    unsigned int epoch = 0;
};

int managed_scratch(const DeviceInfo& di, cudaStream_t s, size_t part_bytes, size_t count_entries,
                    SplitScratch* out) {
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, StreamWorkspace> spaces;
    std::lock_guard<std::mutex> lock(mu);
    StreamWorkspace& w = spaces[{di.device, s}];
    if (part_bytes > w.part_bytes || count_entries > w.count_entries) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
            cudaGetLastError();
            return fail(B2G_ERR_UNSUPPORTED,
                        "split-K workspace must grow (to %zu + %zu bytes) while the stream is being "
                        "captured: run one call of this shape on the stream before capturing",
                        part_bytes, count_entries * sizeof(unsigned long long));
        }
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess)
            return fail(B2G_ERR_CUDA, "split-K workspace: stream synchronize: %s",
                        cudaGetErrorString(e));
        if (part_bytes > w.part_bytes) {
            const size_t bytes = std::max(part_bytes, w.part_bytes * 2);
            if (w.part) cudaFree(w.part);
            w.part = nullptr;
            w.part_bytes = 0;
            if ((e = cudaMalloc(&w.part, bytes)) != cudaSuccess)
                return fail(B2G_ERR_CUDA, "split-K workspace: cudaMalloc(%zu): %s", bytes,
                            cudaGetErrorString(e));
            w.part_bytes = bytes;
        }
        if (count_entries > w.count_entries) {
            const size_t n = std::max(count_entries, w.count_entries * 2);
            if (w.count) cudaFree(w.count);
            w.count = nullptr;
            w.count_entries = 0;
            if ((e = cudaMalloc(&w.count, n * sizeof(unsigned long long))) != cudaSuccess ||
                (e = cudaMemset(w.count, 0, n * sizeof(unsigned long long))) != cudaSuccess)
                return fail(B2G_ERR_CUDA, "split-K counters (%zu): %s", n, cudaGetErrorString(e));
            w.count_entries = n;
        }
    }
    if (++w.epoch == 0) w.epoch = 1;
    *out = SplitScratch{w.part, w.count, w.epoch};
    return B2G_OK;
}

// ---------------------------------------------------------------------------------------
// No-allocation split-K scratch (b2g_gemm_splitk_noalloc)
// ---------------------------------------------------------------------------------------
// For callers that must not allocate device memory at call time (a process that has handed
// all free HBM to its own caching allocator or to a fixed memory budget, or code running in
// a context where an allocation or the stream synchronisation that growing a workspace needs
// is not acceptable). The scratch is this file-scope array, created with the module when the
// library is first used on a device; the library never frees or grows it.
//   [counters: kNoAllocCounters x 8 bytes][FP32 partials: kNoAllocPartBytes]
// The counters must start at zero, and do: a __device__ array without an initializer is
// zero-filled when the module is loaded. They never need clearing afterwards (epoch tags,
// see splitk_arrive); epochs of this scratch start at 1. The partials need no initial value.
constexpr size_t kNoAllocCounters = 32768;                  // (tile, CTA) groups x 8 warps
constexpr size_t kNoAllocPartBytes = (size_t)16 << 20;      // 16 MiB of FP32 partials
constexpr size_t kNoAllocCounterBytes = kNoAllocCounters * sizeof(unsigned long long);
static __device__ __align__(256) unsigned char
    g_b2g_noalloc_scratch[kNoAllocCounterBytes + kNoAllocPartBytes];

// Scratch of one launch from the static array of the current device. The array's address is
// looked up once per device (with that device current, as here). One array per device is
// shared by every call of b2g_gemm_splitk_noalloc on that device, so calls that may overlap
// on the GPU (different streams or host threads) race on it.
int static_scratch(const DeviceInfo& di, size_t part_bytes, size_t count_entries,
                   SplitScratch* out) {
    if (part_bytes > kNoAllocPartBytes || count_entries > kNoAllocCounters)
        return fail(B2G_ERR_ARG,
                    "split-K needs %zu bytes of partials and %zu counters, more than the "
                    "no-allocation scratch holds (%zu bytes, %zu counters): use fewer splits "
                    "or tiles, or b2g_gemm_splitk",
                    part_bytes, count_entries, kNoAllocPartBytes, kNoAllocCounters);
    if (di.device < 0 || di.device >= kMaxDevices)
        return fail(B2G_ERR_ARG, "device %d is beyond the no-allocation scratch table (%d)",
                    di.device, kMaxDevices);
    static std::mutex mu;
    static void* base[kMaxDevices] = {};
    static unsigned int epoch[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (base[di.device] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_b2g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(B2G_ERR_CUDA, "cudaGetSymbolAddress(no-allocation split-K scratch): %s",
                        cudaGetErrorString(e));
        base[di.device] = p;
    }
    if (++epoch[di.device] == 0) epoch[di.device] = 1;
    unsigned char* b = static_cast<unsigned char*>(base[di.device]);
    *out = SplitScratch{reinterpret_cast<float*>(b + kNoAllocCounterBytes),
                        reinterpret_cast<unsigned long long*>(b), epoch[di.device]};
    return B2G_OK;
}

int elementwise_grid(size_t n, int sm_count) {
    const size_t blocks = (n + 255) / 256;
    const size_t cap = (size_t)sm_count * 8;
    return (int)std::max<size_t>(1, std::min(blocks, cap));
}

}  // namespace
}  // namespace b2g

using namespace b2g;

// ---------------------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------------------
namespace b2g {
namespace {

// Everything of b2g_gemm / b2g_gemm_splitk / b2g_gemm_splitk_noalloc after argument
// decoding. `splits`: 0 = automatic, 1 = no split-K, >= 2 = that many K splits (FP32
// accumulation only). `noalloc`: split-K scratch from the static array instead of the
// library-managed per-stream workspace.
int gemm_impl(const void* A, const void* B, void* D, const void* bias, int M, int N, int K,
              long long lda, long long ldb, long long ldd, int b_layout, int acc, int epilogue,
              float alpha, int tile, int stages, int group, int splits, cudaStream_t s,
              bool noalloc = false, const PeerDst* peers = nullptr) {
    static_assert(kMaxPeerDst == kMaxPeers, "peer table sizes");
    if (M < 0 || N < 0 || K < 0)
        return fail(B2G_ERR_ARG, "negative shape M=%d N=%d K=%d", M, N, K);
    if (b_layout != B2G_B_NK && b_layout != B2G_B_KN)
        return fail(B2G_ERR_ARG, "b_layout must be 0 (N x K) or 1 (K x N), got %d", b_layout);
    if (acc != B2G_ACC_F32 && acc != B2G_ACC_F16)
        return fail(B2G_ERR_ARG, "acc must be 0 (FP32) or 1 (FP16), got %d", acc);
    if (epilogue != B2G_EPI_NONE && epilogue != B2G_EPI_BIAS_RELU)
        return fail(B2G_ERR_ARG, "epilogue must be 0 (none) or 1 (bias+ReLU), got %d", epilogue);
    if (tile != B2G_TILE_AUTO && tile != B2G_TILE_128x128 && tile != B2G_TILE_128x256 &&
        tile != B2G_TILE_256x256_2SM && tile != B2G_TILE_128x64 &&
        tile != B2G_TILE_256x512_2SM && tile != B2G_TILE_SWAP_AB && tile != B2G_TILE_256x128_2SM)
        return fail(B2G_ERR_ARG, "tile must be -1 (auto) or 0..6, got %d", tile);
    if (stages != 0 && (stages < 2 || stages > kMaxStages))
        return fail(B2G_ERR_ARG, "stages must be 0 (auto) or 2..%d, got %d", kMaxStages, stages);
    if (group < 0) return fail(B2G_ERR_ARG, "group must be >= 0, got %d", group);
    if (splits < 0) return fail(B2G_ERR_ARG, "splits must be >= 0, got %d", splits);
    if (splits > 1 && acc != B2G_ACC_F32)
        return fail(B2G_ERR_UNSUPPORTED,
                    "split-K sums FP32 partials: it needs FP32 accumulation (acc 0), got acc %d",
                    acc);
    const int npeer = peers ? peers->n : 0;
    if (npeer < 0 || npeer > kMaxPeers)
        return fail(B2G_ERR_ARG, "peer copies of D: 0..%d, got %d", kMaxPeers, npeer);
    if (M == 0 || N == 0) return B2G_OK;
    if (!D) return fail(B2G_ERR_ARG, "D is NULL");
    if (ldd < N) return fail(B2G_ERR_ARG, "ldd (%lld) < N (%d)", ldd, N);
    if (epilogue == B2G_EPI_NONE) bias = nullptr;
    if (npeer > 0) {
        if (N % 8 || ldd % 8 || ((uintptr_t)D & 15))
            return fail(B2G_ERR_ALIGN,
                        "fused all-gather needs N %% 8 == 0, ldd %% 8 == 0 and a 16-byte "
                        "aligned D (N=%d, ldd=%lld)", N, ldd);
        for (int i = 0; i < npeer; ++i)
            if (!peers->ptr[i] || ((uintptr_t)peers->ptr[i] & 15))
                return fail(B2G_ERR_ALIGN, "peer copy %d of D is NULL or not 16-byte aligned", i);
        if (tile == B2G_TILE_SWAP_AB)
            return fail(B2G_ERR_UNSUPPORTED,
                        "the swapped-operand kernel (tile 5) has no fused all-gather");
    }

    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    const bool auto_tile = tile == B2G_TILE_AUTO;
    const int stages_arg = stages, group_arg = group, requested_splits = splits;

    if (K == 0) {  // zero accumulator: only the epilogue remains
        const size_t n = (size_t)M * N;
        for (int i = -1; i < npeer; ++i)
            zero_k_fill_kernel<<<elementwise_grid(n, di.sm_count), 256, 0, s>>>(
                (__half*)(i < 0 ? D : peers->ptr[i]), (const __half*)bias, M, N, ldd, epilogue);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? B2G_OK
                                : fail(B2G_ERR_CUDA, "K == 0 fill launch: %s", cudaGetErrorString(e));
    }
    if (!A || !B) return fail(B2G_ERR_ARG, "A or B is NULL");
    const long long ldb_min = b_layout == B2G_B_NK ? K : N;
    if (lda < K) return fail(B2G_ERR_ARG, "lda (%lld) < K (%d)", lda, K);
    if (ldb < ldb_min) return fail(B2G_ERR_ARG, "ldb (%lld) < %s (%lld)", ldb,
                                   b_layout == B2G_B_NK ? "K" : "N", ldb_min);
    if (((uintptr_t)A & 15) || ((uintptr_t)B & 15))
        return fail(B2G_ERR_ALIGN, "A and B must be 16-byte aligned (TMA)");
    if ((lda % 8) || (ldb % 8))
        return fail(B2G_ERR_ALIGN,
                    "lda (%lld) and ldb (%lld) must be multiples of 8 elements: TMA row "
                    "strides are multiples of 16 bytes (pad the leading dimension)",
                    lda, ldb);

    // One CTA per 128 x 128 tile when either side is small (no half-empty 256-row pair
    // tiles for skinny M, fewer idle columns for narrow N), or when 256 x 256 pair tiles would
    // occupy under half of the pairs while 128 x 128 tiles fit one wave (measured on B200:
    // 1024^3 245 -> 258 TFLOP/s, 512^3 38 -> 42; the pair kernel's tail slices reload A);
    // else 2-CTA 256 x 256 pairs.
    bool pair_split = false;
    if (tile == B2G_TILE_AUTO) {
        const long long pair_tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
        const long long small_tiles = (long long)((M + 127) / 128) * ((N + 127) / 128);
        const bool sparse_pairs = 2 * pair_tiles < di.sm_count / 2 && small_tiles <= di.sm_count;
        // Pair tiles that would fill between a quarter and a half of the pair clusters, with
        // long K: two K splits per tile, reduced inside a cluster of the two pairs, fill the
        // GPU with pairs, whose L2 -> SM traffic per FLOP is half that of 128 x 128 tiles
        // (measured on B200: 512 x 4096 x 4096 22.7 us on 128 x 128 tiles -> 20.7 us).
        pair_split = sparse_pairs && 4 * pair_tiles > di.sm_count / 2 && K >= 2048 &&
                     acc == B2G_ACC_F32 && requested_splits == 0 && !noalloc && npeer == 0 &&
                     b_layout == B2G_B_NK && csplit_enabled();
        tile = (N <= 128 || M <= 128 || (sparse_pairs && !pair_split)) ? B2G_TILE_128x128
                                                                      : B2G_TILE_256x256_2SM;
        // 256 x 512 pair tiles when every pair gets enough of them to amortise the half-1
        // hand-over at each tile start: K >= 4096, >= 3.5 waves of wide tiles and >= 320
        // k-blocks of wide tiles per pair; then the wide tile's quarter less L2 traffic per
        // FLOP wins (measured on B200, device time: 8192^3 1446 -> 1503, 16384^3 1253 -> 1310,
        // 4096 x 32768 x 8192 1443 -> 1512 TFLOP/s; 6144^3 374.8 -> 354.7 us, 8192 x 8192 x 4096
        // 442.7 -> 427.0 us; 6144 x 6144 x 4096, 249 k-blocks per pair, 221.7 -> 253.2 us and
        // 5120^3, 2.7 waves, 203.8 -> 219.4 us stay on 256 x 256 tiles).
        const long long wide_tiles = (long long)((M + 255) / 256) * ((N + 511) / 512);
        const long long pairs = di.sm_count / 2;
        if (tile == B2G_TILE_256x256_2SM && K >= 4096 && 2 * wide_tiles >= 7 * pairs &&
            wide_tiles * ((K + 63) / 64) >= 320 * pairs)
            tile = B2G_TILE_256x512_2SM;
        // Tiny M with N wide enough that 128-column blocks alone give ~one CTA per SM (no
        // split-K needed): the swapped-operand kernel skips the 128-row tile's padding
        // (measured on B200: 16 x 16384 x 4096 77.8 -> 84.7 TFLOP/s; with N = 4096 its 32
        // CTAs are slower than 128 x 128 tiles with split-K, so it is not used there).
        const long long n_blocks = (N + 127) / 128;
        if (M <= 32 && b_layout == B2G_B_NK && requested_splits <= 1 && npeer == 0 &&
            2 * n_blocks > di.sm_count && 3 * n_blocks >= 2LL * di.sm_count)
            tile = B2G_TILE_SWAP_AB;
    }
    if (tile == B2G_TILE_SWAP_AB) {
        if (b_layout != B2G_B_NK)
            return fail(B2G_ERR_UNSUPPORTED, "the swapped-operand kernel takes B as N x K only");
        if (splits > 1)
            return fail(B2G_ERR_UNSUPPORTED, "split-K is not built for the swapped-operand kernel");
        GemmParams p{};
        p.M = M;
        p.N = N;
        p.K = K;
        p.num_kb = (K + kBK - 1) / kBK;
        p.group = group;
        p.acc_f16 = acc == B2G_ACC_F16;
        p.epilogue = epilogue;
        p.alpha = alpha;
        p.bias = (const __half*)bias;
        p.D = (__half*)D;
        p.ldd = ldd;
        p.timeout_ns = wait_timeout_ns();
        switch (swap_mt_for(M, N, di.sm_count)) {
            case 16: return launch_swap<16>(A, B, M, N, K, lda, ldb, p, stages, di, s);
            case 32: return launch_swap<32>(A, B, M, N, K, lda, ldb, p, stages, di, s);
            default: return launch_swap<64>(A, B, M, N, K, lda, ldb, p, stages, di, s);
        }
    }
    const TileGeom g = geom(tile);
    const int epi_boxes = epi_boxes_for((K + kBK - 1) / kBK);
    // A box rows: all of M in one 1-CTA tile -> load (and stage) only round_up(M, 8) rows per
    // k-block
    const int a_rows = (g.ctas == 1 && M <= g.bm) ? std::min(g.box_a, (M + 7) / 8 * 8) : g.box_a;
    const int max_st = max_stages_for(tile, di.smem_optin, epi_boxes, a_rows);
    if (stages == 0) stages = max_st;
    if (smem_needed(tile, stages, epi_boxes, a_rows) > (size_t)di.smem_optin)
        return fail(B2G_ERR_SMEM, "smem over per-block opt-in limit: %zu > %d (tile %d, %d stages)",
                    smem_needed(tile, stages, epi_boxes, a_rows), di.smem_optin, tile, stages);
    size_t smem = smem_request(tile, stages, di, epi_boxes, a_rows);

    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.tiles_m = (M + g.bm - 1) / g.bm;
    p.tiles_n = (N + g.bn - 1) / g.bn;
    const long long nt = (long long)p.tiles_m * p.tiles_n;
    if (nt > 0x7fffffffLL) return fail(B2G_ERR_ARG, "too many tiles (%lld)", nt);
    p.num_tiles = (int)nt;
    p.num_kb = (K + kBK - 1) / kBK;
    p.stage_tx = (uint32_t)(a_rows + g.box_b) * kBK * 2;
    p.a_stage_bytes = (uint32_t)a_rows * kBK * 2;
    p.group = group > 0 ? group : auto_group(g, p.tiles_m, K);
    p.stages = stages;
    const bool b_mn = b_layout == B2G_B_KN;
    const bool wide = tile == B2G_TILE_256x512_2SM;
    p.idesc = idesc_f16(g.bm, std::min(g.bn, kPairBN), acc == B2G_ACC_F32, b_mn);
    p.acc_f16 = acc == B2G_ACC_F16;
    p.epilogue = epilogue;
    p.alpha = alpha;
    p.bias = (const __half*)bias;
    p.D = (__half*)D;
    p.ldd = ldd;
    p.d_tma = (((uintptr_t)D & 15) == 0) && (ldd % 8 == 0);
    p.peers.n = npeer;
    for (int i = 0; i < npeer; ++i) p.peers.d[i] = (__half*)peers->ptr[i];
    p.b_mn_major = b_mn ? 1 : 0;
    p.dp_tiles = p.num_tiles;
    p.tail_split = 1;
    p.num_units = p.num_tiles;
    p.idesc_tail = p.idesc;
    // split-K: tiles that fill under half of the SMs (pairs) get their K range split
    const int concurrent = g.ctas == 2 ? max_pair_clusters(di, smem) : di.sm_count;
    if (splits == 0)
        splits = pair_split ? 2
                            : acc == B2G_ACC_F32 ? splitk_auto(p.num_tiles, concurrent, p.num_kb, g.ctas)
                                                 : 1;
    if (splits > p.num_kb)
        return fail(B2G_ERR_ARG, "splits (%d) > k-blocks of 64 (%d)", splits, p.num_kb);
    if (wide && splits > 1)
        return fail(B2G_ERR_UNSUPPORTED, "split-K is not built for the 256 x 512 tile (tile 4)");
    if ((long long)p.num_tiles * splits > 0x7fffffffLL)
        return fail(B2G_ERR_ARG, "too many work units (%d tiles x %d splits)", p.num_tiles, splits);
    // Small problems on 128 x 128 tiles that leave more than half the SMs idle and gain
    // nothing from split-K (short K) take 128 x 64 tiles instead (auto tile and split only;
    // measured on B200: 512^3 42.0 -> 44.9, 1024^3 242.8 -> 255.4 TFLOP/s).
    if (auto_tile && requested_splits == 0 && splits == 1 && tile == B2G_TILE_128x128 &&
        2LL * p.num_tiles <= di.sm_count)
        return gemm_impl(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue, alpha,
                         B2G_TILE_128x64, stages_arg, group_arg, requested_splits, s, noalloc,
                         peers);
    p.splits = splits;
    p.num_units = p.num_tiles * splits;
    // Split-K of 1-CTA tiles is reduced inside clusters of `splits` CTAs through distributed
    // shared memory when the receive slots fit beside a ring of at least two stages (measured
    // on B200: the workspace's partial stores, release-ordered arrival and L2 re-reads cost
    // more than the split mainloop they serve at decode shapes). b2g_gemm_splitk_noalloc
    // keeps the workspace path on its static scratch; both reductions give the same bits.
    // (1-CTA tiles: clusters of S <= 8 CTAs; 2-CTA 256 x 256 and 256 x 128 tiles: S <= 4
    // pairs, 8 CTAs; the receive slots of the CTA's 128 x min(BN, 256) accumulator overlay the
    // ring, which must hold them)
    // Where the receive slots go (measured on B200, N = K = 4096): on 1-CTA tiles their own
    // shared memory when that still leaves a ring of at least 4 stages -- a split then sends as
    // soon as its own accumulator is final (M = 128: 14.7 us, vs 15.4 us with 6 stages and the
    // slots over the ring; M = 1: 12.5 vs 13.3 us); on pair tiles, whose mainloop needs the
    // deeper ring more, over the drained ring unless their own memory costs no stage (M = 512
    // on 256 x 256 pairs: 20.7 us over the ring with 6 stages vs 22.2 us with 4).
    if (splits > 1 && !noalloc && !wide && splits * g.ctas <= 8 && csplit_enabled()) {
        const uint32_t recv = csplit_recv_bytes(std::min(g.bn, kPairBN), splits);
        const size_t stage_b = (size_t)a_rows * kBK * 2 + (size_t)g.box_b * kBK * 2;
        int st_own = stages;
        if (stages_arg == 0)
            while (st_own > 2 && smem_needed(tile, st_own, epi_boxes, a_rows) + recv >
                                     (size_t)di.smem_optin)
                --st_own;
        const bool own = smem_needed(tile, st_own, epi_boxes, a_rows) + recv <=
                             (size_t)di.smem_optin &&
                         (st_own == stages || (g.ctas == 1 && st_own >= 4));
        if (own || recv <= (size_t)stages * stage_b) {
            const size_t req = own ? std::max(smem_needed(tile, st_own, epi_boxes, a_rows) + recv,
                                              (size_t)di.smem_per_sm / 2 + 1024)
                                   : smem;
            if (int rc = ensure_kernel_attrs(tile, di, npeer > 0 ? kVarPeers : kVarCsplit))
                return rc;
            if (cluster_fits(di, tile, splits * g.ctas, gemm_threads(8), req, npeer > 0)) {
                p.csplit = 1;
                p.recv_ring = own ? 0 : 1;
                p.recv_bytes = recv;
                if (own) {
                    stages = st_own;
                    p.stages = st_own;
                    smem = req;
                }
            }
        }
    }
    if (splits > 1 && !p.csplit) {
        const size_t part = (size_t)p.num_tiles * splits * g.ctas * 128 * g.bn * sizeof(float);
        const size_t counters = (size_t)p.num_tiles * g.ctas * kMaxEpiWarps;
        SplitScratch sc{};
        if (int rc = noalloc ? static_scratch(di, part, counters, &sc)
                             : managed_scratch(di, s, part, counters, &sc))
            return rc;
        p.ws_part = sc.part;
        p.ws_count = sc.count;
        p.epoch = sc.epoch;
    }
    if (g.ctas == 2 && splits == 1) {
        // cut the tiles of the last, partial wave into column slices (see pair_unit)
        const int clusters = max_pair_clusters(di, smem);
        const int rest = p.num_tiles % clusters;
        // K x N B loads 64-column boxes: a slice needs >= 64 columns per CTA
        // (256 x 128 tiles are not sliced: their 64-column slices would reload A for little)
        const int max_split = g.bn == 128 ? 1 : b_mn ? std::max(1, g.bn / 128) : 4;
        const int split = rest ? tail_split_for(rest, clusters, max_split, wide) : 1;
        if (split > 1) {
            p.dp_tiles = p.num_tiles - rest;
            p.tail_split = split;
            p.num_units = p.dp_tiles + rest * split;
            p.idesc_tail = idesc_f16(g.bm, std::min(g.bn / split, kPairBN), acc == B2G_ACC_F32,
                                     b_mn);
        }
    }
    p.timeout_ns = wait_timeout_ns();

    CUtensorMap tmA, tmB;
    if (int rc = make_tmap(&tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, kBK,
                           (uint32_t)a_rows, "A"))
        return rc;
    // B: N x K in 128-row x 64-k boxes, or K x N (MN-major) either in one 3D box of all the
    // 64-column groups a CTA loads per stage (N % 64 == 0) or in 64-column x 64-k-row boxes
    // (columns per CTA and stage: BN on one CTA, min(tile width, 256) / 2 per CTA of a pair)
    const auto kn_groups = [&](int width) {
        return (uint32_t)((g.ctas == 2 ? std::min(width, kPairBN) / 2 : width) / 64);
    };
    if (b_mn && N % 64 == 0 && kn3d_enabled()) {
        if (make_tmap_kn3d(&tmB, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, kn_groups(g.bn)) ==
            B2G_OK)
            p.b_kn3d = 1;
        else
            clear_error();  // not encodable here: the 2D boxes below
    }
    if (!p.b_kn3d)
        if (int rc = b_mn ? make_tmap(&tmB, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, kBK, "B")
                          : make_tmap(&tmB, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, kBK,
                                      g.box_b, "B"))
            return rc;
    CUtensorMap tmBt = tmB;  // B boxes of the tail slices (min(width, 256) / 2 rows per CTA)
    if (p.tail_split > 1 && p.b_kn3d) {
        if (int rc = make_tmap_kn3d(&tmBt, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb,
                                    kn_groups(g.bn / p.tail_split)))
            return rc;
    } else if (p.tail_split > 1 && !b_mn) {
        if (int rc = make_tmap(&tmBt, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, kBK,
                               (uint32_t)(std::min(g.bn / p.tail_split, kPairBN) / 2), "B tail"))
            return rc;
    }
    CUtensorMap tmD = tmA;  // D in 32-row x 64-column boxes (unused without d_tma)
    if (p.d_tma)
        if (int rc = make_tmap(&tmD, D, (uint64_t)N, (uint64_t)M, (uint64_t)ldd, 64, 32, "D"))
            return rc;
    const int ctas_at_once = g.ctas == 2 ? 2 * max_pair_clusters(di, smem) : di.sm_count;
    const int epi_warps = epi_warps_for(p.num_kb, p.splits, wide,
                                        (long long)p.num_units * g.ctas <= ctas_at_once);
    p.epi_bufs = std::max(1, std::min(kMaxEpiBufs, epi_boxes / epi_warps));
    return launch_gemm(tile, tmA, tmB, tmBt, tmD, p, di, smem, s, epi_warps);
}

}  // namespace
}  // namespace b2g

namespace b2g {
int allgather_push(const void* src, int rows, int N, long long ldd, void* const* dst, int ndst,
                   void* stream) {
    if (ndst < 1 || ndst > kMaxGatherDst)
        return fail(B2G_ERR_ARG, "all-gather destinations: 1..%d, got %d", kMaxGatherDst, ndst);
    if (rows <= 0 || N <= 0) return B2G_OK;
    GatherDst d{};
    d.n = ndst;
    for (int i = 0; i < ndst; ++i) d.d[i] = (__half*)dst[i];
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    const int grid = std::min(rows, 4 * di.sm_count);
    allgather_push_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const __half*)src, rows, N / 8,
                                                                   ldd, d);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? B2G_OK
                            : fail(B2G_ERR_CUDA, "all-gather push launch: %s", cudaGetErrorString(e));
}

int gemm_to_peers(const void* A, const void* B, void* D, const void* bias, int M, int N, int K,
                  long long lda, long long ldb, long long ldd, int b_layout, int acc,
                  int epilogue, float alpha, int tile, int stages, int group, void* stream,
                  const PeerDst& peers) {
    return gemm_impl(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue, alpha, tile,
                     stages, group, 0, (cudaStream_t)stream, false, &peers);
}
}  // namespace b2g

B2G_EXPORT int b2g_gemm(const void* A, const void* B, void* D, const void* bias, int M, int N,
                        int K, long long lda, long long ldb, long long ldd, int b_layout,
                        int acc, int epilogue, float alpha, int tile, int stages, int group,
                        void* stream) {
    clear_error();
    return gemm_impl(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue, alpha, tile,
                     stages, group, 0, (cudaStream_t)stream);
}

B2G_EXPORT int b2g_gemm_splitk(const void* A, const void* B, void* D, const void* bias, int M,
                               int N, int K, long long lda, long long ldb, long long ldd,
                               int b_layout, int acc, int epilogue, float alpha, int tile,
                               int stages, int group, int splits, void* stream) {
    clear_error();
    return gemm_impl(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue, alpha, tile,
                     stages, group, splits, (cudaStream_t)stream);
}

B2G_EXPORT int b2g_gemm_splitk_noalloc(const void* A, const void* B, void* D, const void* bias,
                                       int M, int N, int K, long long lda, long long ldb,
                                       long long ldd, int b_layout, int acc, int epilogue,
                                       float alpha, int tile, int stages, int group, int splits,
                                       void* stream) {
    clear_error();
    return gemm_impl(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue, alpha, tile,
                     stages, group, splits, (cudaStream_t)stream, true);
}

B2G_EXPORT int b2g_config_info(int tile, int stages, int* threads, int* regs, int* smem_bytes,
                               int* ctas_per_sm, int* tmem_cols, int* stages_used) {
    clear_error();
    if (tile == B2G_TILE_AUTO) tile = B2G_TILE_256x256_2SM;
    if (tile != B2G_TILE_128x128 && tile != B2G_TILE_128x256 && tile != B2G_TILE_256x256_2SM &&
        tile != B2G_TILE_128x64 && tile != B2G_TILE_256x512_2SM && tile != B2G_TILE_SWAP_AB &&
        tile != B2G_TILE_256x128_2SM)
        return fail(B2G_ERR_UNSUPPORTED, "tile %d is not built", tile);
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    if (stages == 0) stages = max_stages_for(tile, di.smem_optin);
    if (stages < 2 || stages > kMaxStages)
        return fail(B2G_ERR_ARG, "stages must be 2..%d", kMaxStages);
    const size_t need = smem_needed(tile, stages);
    if (need > (size_t)di.smem_optin)
        return fail(B2G_ERR_SMEM, "smem over per-block opt-in limit: %zu > %d", need, di.smem_optin);
    if (int rc = ensure_kernel_attrs(tile, di)) return rc;
    const size_t smem = smem_request(tile, stages, di);
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel_ptr(tile));
    if (e != cudaSuccess)
        return fail(B2G_ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel_ptr(tile), kMaxThreads,
                                                      smem) != cudaSuccess) {
        cudaGetLastError();
        occ = 0;
    }
    if (threads) *threads = kMaxThreads;
    if (regs) *regs = fa.numRegs;
    if (smem_bytes) *smem_bytes = (int)need;
    if (ctas_per_sm) *ctas_per_sm = occ;
    if (tmem_cols) *tmem_cols = tile == B2G_TILE_SWAP_AB ? 2 * 64 : std::min(2 * geom(tile).bn, 512);
    if (stages_used) *stages_used = stages;
    return B2G_OK;
}

B2G_EXPORT int b2g_last_launch(int* grid, int* threads, int* tile, int* stages, int* units,
                               int* splits) {
    clear_error();
    const LaunchRecord r = g_last_launch;
    if (r.grid == 0) return fail(B2G_ERR_ARG, "no GEMM kernel launched on this host thread yet");
    if (grid) *grid = r.grid;
    if (threads) *threads = r.threads;
    if (tile) *tile = r.tile;
    if (stages) *stages = r.stages;
    if (units) *units = r.units;
    if (splits) *splits = r.splits;
    return B2G_OK;
}

B2G_EXPORT int b2g_last_launch_cluster(int* cluster_ctas) {
    clear_error();
    const LaunchRecord r = g_last_launch;
    if (r.grid == 0) return fail(B2G_ERR_ARG, "no GEMM kernel launched on this host thread yet");
    if (cluster_ctas) *cluster_ctas = r.cluster;
    return B2G_OK;
}

B2G_EXPORT int b2g_last_launch_variant(int* variant) {
    clear_error();
    const LaunchRecord r = g_last_launch;
    if (r.grid == 0) return fail(B2G_ERR_ARG, "no GEMM kernel launched on this host thread yet");
    if (variant) *variant = r.variant;
    return B2G_OK;
}

// ---------------------------------------------------------------------------------------
// Status word
// ---------------------------------------------------------------------------------------
B2G_EXPORT int b2g_sync_status(void* stream) {
    clear_error();
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "stream synchronize: %s", cudaGetErrorString(e));
    unsigned int word = 0;
    e = cudaMemcpyFromSymbol(&word, g_b2g_status, sizeof(word));
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "read status word: %s", cudaGetErrorString(e));
    if (word == 0) return B2G_OK;
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(g_b2g_status, &zero, sizeof(zero));
    return fail(B2G_ERR_TIMEOUT,
                "device wait gave up (status 0x%x:%s%s%s%s%s%s%s); the kernel unwound and "
                "returned",
                word, (word & kErrWaitProducer) ? " producer" : "", (word & kErrWaitMma) ? " mma" : "",
                (word & kErrWaitEpilogue) ? " epilogue" : "",
                (word & kErrWaitSelftest) ? " selftest" : "", (word & kErrWaitDrain) ? " drain" : "",
                (word & kErrWaitProbe) ? " probe" : "",
                (word & kErrSplitCounter) ? " split-K counter" : "");
}

#ifdef B2G_INSTRUMENT
// Instrumented builds only: copy out (n <= 1024 CTAs x 8 slots) and clear the wait-time
// counters of sm100_ptx.cuh.
B2G_EXPORT int b2g_instr_read(unsigned long long* out, int n_ctas) {
    const size_t bytes = sizeof(unsigned long long) * kInstrSlots * (size_t)n_ctas;
    if (cudaMemcpyFromSymbol(out, g_b2g_instr, bytes) != cudaSuccess) return B2G_ERR_CUDA;
    static unsigned long long zeros[1024][kInstrSlots];
    return cudaMemcpyToSymbol(g_b2g_instr, zeros, sizeof(zeros)) == cudaSuccess ? B2G_OK
                                                                                : B2G_ERR_CUDA;
}
// Copy out the marks of the first n_ctas (<= 1024) CTAs of the most recent launch:
// 2 x kTlMarks per CTA (global timer, then clock64).
B2G_EXPORT int b2g_instr_timeline(unsigned long long* out, int n_ctas) {
    return cudaMemcpyFromSymbol(out, g_b2g_tl,
                                sizeof(unsigned long long) * 2 * kTlMarks * (size_t)n_ctas) ==
                   cudaSuccess
               ? B2G_OK
               : B2G_ERR_CUDA;
}
#endif

B2G_EXPORT int b2g_kernel_clock(double* sm_mhz, double* cta0_us) {
    clear_error();
    unsigned long long c[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpyFromSymbol(c, g_b2g_clock, sizeof(c));
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "read clock telemetry: %s", cudaGetErrorString(e));
    if (c[1] <= c[0] || c[3] <= c[2]) return fail(B2G_ERR_ARG, "no completed GEMM launch recorded");
    const double ns = (double)(c[1] - c[0]);
    if (sm_mhz) *sm_mhz = (double)(c[3] - c[2]) / ns * 1e3;
    if (cta0_us) *cta0_us = ns * 1e-3;
    return B2G_OK;
}

B2G_EXPORT int b2g_selftest_wait_timeout(unsigned timeout_us, void* stream) {
    clear_error();
    if (timeout_us < 1 || timeout_us > 2000000)
        return fail(B2G_ERR_ARG, "timeout_us must be 1..2000000, got %u", timeout_us);
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(1000ull * timeout_us);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "selftest launch: %s", cudaGetErrorString(e));
    return b2g_sync_status(stream);
}

// ---------------------------------------------------------------------------------------
// Auxiliary kernels
// ---------------------------------------------------------------------------------------
B2G_EXPORT int b2g_max_rel_diff(const void* x, const void* y, size_t n, float* out_dev,
                                void* stream) {
    clear_error();
    if (!out_dev || (n && (!x || !y))) return fail(B2G_ERR_ARG, "NULL pointer");
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(out_dev, 0, sizeof(float), s);
    if (e == cudaSuccess && n) {
        max_rel_diff_kernel<<<elementwise_grid(n, di.sm_count), 256, 0, s>>>(
            (const __half*)x, (const __half*)y, n, out_dev);
        e = cudaGetLastError();
    }
    return e == cudaSuccess ? B2G_OK : fail(B2G_ERR_CUDA, "max_rel_diff: %s", cudaGetErrorString(e));
}

B2G_EXPORT int b2g_bias_relu(void* D, const void* bias, int M, int N, long long ldd, float alpha,
                             void* stream) {
    clear_error();
    if (M < 0 || N < 0 || ldd < N) return fail(B2G_ERR_ARG, "bad shape M=%d N=%d ldd=%lld", M, N, ldd);
    if (M == 0 || N == 0) return B2G_OK;
    if (!D) return fail(B2G_ERR_ARG, "D is NULL");
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    const size_t n = (size_t)M * N;
    bias_relu_kernel<<<elementwise_grid(n, di.sm_count), 256, 0, (cudaStream_t)stream>>>(
        (__half*)D, (const __half*)bias, M, N, ldd, alpha);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? B2G_OK : fail(B2G_ERR_CUDA, "bias_relu: %s", cudaGetErrorString(e));
}

B2G_EXPORT int b2g_probe_hbm(const void* src, void* dst, size_t bytes, int reps, void* stream,
                             double* gbs) {
    clear_error();
    if (!src || !dst || !gbs || reps < 1 || bytes < 16 || (bytes & 15) ||
        (((uintptr_t)src | (uintptr_t)dst) & 15))
        return fail(B2G_ERR_ARG, "hbm probe needs 16-byte aligned buffers, bytes %% 16 == 0, reps >= 1");
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t n16 = bytes / 16;
    const int grid = di.sm_count * 4;
    for (int w = 0; w < 3; ++w)
        hbm_copy_kernel<<<grid, 512, 0, s>>>((const uint4*)src, (uint4*)dst, n16);
    cudaEvent_t t0, t1;
    cudaEventCreate(&t0);
    cudaEventCreate(&t1);
    cudaEventRecord(t0, s);
    for (int r = 0; r < reps; ++r)
        hbm_copy_kernel<<<grid, 512, 0, s>>>((const uint4*)src, (uint4*)dst, n16);
    cudaEventRecord(t1, s);
    cudaError_t e = cudaEventSynchronize(t1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t0, t1);
    cudaEventDestroy(t0);
    cudaEventDestroy(t1);
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "hbm probe: %s", cudaGetErrorString(e));
    *gbs = 2.0 * (double)bytes * reps / (ms * 1e-3) / 1e9;  // each byte read once, written once
    return B2G_OK;
}

// ---------------------------------------------------------------------------------------
// tcgen05 issue-rate probe
// ---------------------------------------------------------------------------------------
B2G_EXPORT int b2g_probe_tcgen05(int kind, int cta_group, int n, int iters,
                                 double* flop_per_clk_sm, long long* cycles_out) {
    clear_error();
    if (kind < 0 || kind > 3) return fail(B2G_ERR_ARG, "kind must be 0..3, got %d", kind);
    if (cta_group != 1 && cta_group != 2)
        return fail(B2G_ERR_ARG, "cta_group must be 1 or 2, got %d", cta_group);
    if (n < 16 || n > 256 || n % 16) return fail(B2G_ERR_ARG, "n must be 16..256, step 16");
    if (iters < 1 || iters > (1 << 24)) return fail(B2G_ERR_ARG, "iters must be 1..2^24");
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    // one CTA per SM (cta_group 1) or one 2-CTA cluster per pair of SMs (cta_group 2)
    const int blocks = cta_group == 1 ? di.sm_count : 2 * (di.sm_count / 2);
    const int timed = cta_group == 1 ? blocks : blocks / 2;
    long long* dcyc = nullptr;
    cudaError_t e = cudaMalloc(&dcyc, sizeof(long long) * timed);
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "probe cudaMalloc: %s", cudaGetErrorString(e));
    e = cudaMemset(dcyc, 0, sizeof(long long) * timed);
    const uint32_t idesc = idesc_probe(kind, cta_group == 1 ? 128 : 256, n);
    const unsigned long long tmo = wait_timeout_ns();
    auto run = [&](auto kern) -> cudaError_t {
        cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kProbeSmem);
        if (r != cudaSuccess) return r;
        for (int w = 0; w < 4; ++w) kern<<<blocks, kProbeThreads, kProbeSmem>>>(idesc, iters, dcyc, tmo);
        return cudaDeviceSynchronize();
    };
    if (e == cudaSuccess) {
        if (cta_group == 1) {
            switch (kind) {
                case kProbeF16F32: e = run(probe_tcgen05_kernel<kProbeF16F32>); break;
                case kProbeF16F16: e = run(probe_tcgen05_kernel<kProbeF16F16>); break;
                case kProbeI8: e = run(probe_tcgen05_kernel<kProbeI8>); break;
                default: e = run(probe_tcgen05_kernel<kProbeE4M3>); break;
            }
        } else {
            switch (kind) {
                case kProbeF16F32: e = run(probe_tcgen05_pair_kernel<kProbeF16F32>); break;
                case kProbeF16F16: e = run(probe_tcgen05_pair_kernel<kProbeF16F16>); break;
                case kProbeI8: e = run(probe_tcgen05_pair_kernel<kProbeI8>); break;
                default: e = run(probe_tcgen05_pair_kernel<kProbeE4M3>); break;
            }
        }
    }
    long long best = -1;
    if (e == cudaSuccess) {
        long long* h = new long long[timed];
        e = cudaMemcpy(h, dcyc, sizeof(long long) * timed, cudaMemcpyDeviceToHost);
        for (int b = 0; b < timed && e == cudaSuccess; ++b)
            if (h[b] > 0 && (best < 0 || h[b] < best)) best = h[b];  // least-perturbed SM
        delete[] h;
    }
    cudaFree(dcyc);
    if (e != cudaSuccess) return fail(B2G_ERR_CUDA, "probe: %s", cudaGetErrorString(e));
    if (int rc = b2g_sync_status(nullptr)) return rc;
    if (best <= 0) return fail(B2G_ERR_TIMEOUT, "probe produced no timing");
    // FLOP of one MMA: 2 x M x N x K, M = 128 per SM (the pair's M = 256 spans two SMs)
    const double flop = 2.0 * 128.0 * n * probe_mma_k(kind) * (double)iters;
    if (flop_per_clk_sm) *flop_per_clk_sm = flop / (double)best;
    if (cycles_out) *cycles_out = best;
    return B2G_OK;
}
