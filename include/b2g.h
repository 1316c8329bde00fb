/*
 * b2g.h -- C-ABI of the B200 (sm_100a) FP16 tensor-core GEMM.
 *
 * D = A * B with FP16 inputs, FP32 or FP16 accumulation, FP16 output, optionally fused
 * alpha*acc + bias + ReLU. Kernels are hand-written for sm_100a: TMA tile loads into an
 * mbarrier-guarded shared-memory ring, tcgen05.mma with accumulators in tensor memory,
 * and a persistent, warp-specialised tile scheduler.
 *
 * The reference (a single-file sm_89 benchmark) has no library ABI; its boundary is the
 * kernel launch inside its CLI. Each entry point below names the reference code it
 * replaces (paths relative to the reference project root).
 *
 * Conventions
 *   - Plain pointers and sizes only. FP16 data is IEEE binary16 (uint16_t bit patterns).
 *   - Device pointers are caller-owned; no entry point keeps them after it returns.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Layouts (reference src/gemm_bench.cu:8-15):
 *       A: M x K row-major, leading dimension lda >= K
 *       B: b_layout B2G_B_NK: N x K row-major (ldb >= K), the reference's "TN" layout
 *          b_layout B2G_B_KN: K x N row-major (ldb >= N; not in the reference, whose kernel
 *          takes only the TN layout): read as an MN-major operand, same results bit for bit
 *       D: M x N row-major, ldd >= N
 *   - Launch entry points are asynchronous and never call exit(). They return a b2g_status;
 *     b2g_last_error() gives the message of the last failure on the calling thread.
 *     A device-side failure (a bounded wait that ran out) is reported by b2g_sync_status().
 */
#ifndef B2G_H
#define B2G_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum b2g_status {
    B2G_OK = 0,
    B2G_ERR_ARG = 1,         /* bad shape or flag value                                   */
    B2G_ERR_ALIGN = 2,       /* pointer / leading dimension breaks the 16-byte TMA rule   */
    B2G_ERR_UNSUPPORTED = 3, /* configuration not built (reference: pick() -> nullptr)    */
    B2G_ERR_SMEM = 4,        /* over the shared-memory opt-in limit (reference: SKIP row) */
    B2G_ERR_CUDA = 5,        /* a CUDA runtime / driver call failed                       */
    B2G_ERR_TIMEOUT = 6,     /* a device-side wait hit its limit; the kernel returned     */
    B2G_ERR_NO_DEVICE = 7,   /* no sm_100 device is current                               */
    B2G_ERR_LIBRARY = 8      /* cuBLAS (comparison column only) failed                    */
};

enum { B2G_B_NK = 0, B2G_B_KN = 1 };              /* B operand layout               */
enum { B2G_ACC_F32 = 0, B2G_ACC_F16 = 1 };        /* accumulator type               */
enum { B2G_EPI_NONE = 0, B2G_EPI_BIAS_RELU = 1 }; /* epilogue                       */

/* Tile configurations (the `tile` argument). Replaces the reference's TileCfg<0..4>
 * (src/gemm_bench.cu:413-425), which are Ada warp tilings with no meaning on tcgen05.
 *   B2G_TILE_128x128   : one CTA, UMMA 128x128x16, TMEM 2 x 128 columns
 *   B2G_TILE_128x256   : one CTA, UMMA 128x256x16, TMEM 2 x 256 columns
 *   B2G_TILE_128x64    : one CTA, UMMA 128x64x16, TMEM 2 x 64 columns (small problems:
 *                        twice the tiles of 128x128)
 *   B2G_TILE_256x512_2SM : a 2-CTA cluster computing a 256 x 512 tile as two UMMA
 *                        256x256x16 halves (all 512 TMEM columns, halves released to the
 *                        next tile separately); a quarter less L2 traffic per FLOP than
 *                        256x256 (large problems; no split-K)
 *   B2G_TILE_SWAP_AB   : small M (decode): one CTA per 128 columns of D x MT rows, UMMA
 *                        128 x MT x 16 with B's rows on the 128 side (MT = 16, 32 or 64,
 *                        from M and N); B as N x K only, no split-K
 *   B2G_TILE_256x128_2SM : a 2-CTA cluster, UMMA 256x128x16: per CTA 16 KiB of A + 8 KiB of
 *                        B per k-block for 128 x 128 outputs (a quarter less than one CTA
 *                        per 128 x 128 tile)
 *   B2G_TILE_256x256_2SM : a 2-CTA cluster (cta_group::2), UMMA 256x256x16, each CTA loads
 *                        its own 128 rows of A and 128 rows of B (no multicast)
 *   B2G_TILE_AUTO      : chosen from the shape                                           */
enum {
    B2G_TILE_128x128 = 0,
    B2G_TILE_128x256 = 1,
    B2G_TILE_256x256_2SM = 2,
    B2G_TILE_128x64 = 3,
    B2G_TILE_256x512_2SM = 4,
    B2G_TILE_SWAP_AB = 5,
    B2G_TILE_256x128_2SM = 6,
    B2G_TILE_AUTO = -1
};

/* ---------------------------------------------------------------------------------------
 * GEMM. Replaces gemm_kernel<BM,BN,BK,WM,WN,STAGES,LAYOUT>(A, B, D, bias, M, N, K, alpha,
 * group) (src/gemm_bench.cu:213-217) as launched by run_cfg (src/gemm_bench.cu:480-488)
 * and selected by pick(tile, layout, stages) (src/gemm_bench.cu:596-605). The reference's
 * compile-time switches FUSE_EPILOGUE and ACC_F16 (src/gemm_bench.cu:31-47) are the
 * runtime arguments `epilogue` and `acc` here.
 *
 *   bias     : N FP16 values, read only when epilogue == B2G_EPI_BIAS_RELU (may be NULL)
 *   alpha    : epilogue scale (reference passes 1.0f, src/gemm_bench.cu:482)
 *   tile     : B2G_TILE_* ; stages: shared-memory ring depth, 0 = deepest that fits
 *   group    : L2 rasterization, `group` M-tiles walked column-major (1 = row-major),
 *              same mapping as src/gemm_bench.cu:237-250; 0 = the largest band whose A
 *              rows fill ~30% of the L2 (measured best on B200)
 * Requirements: A, B 16-byte aligned; lda, ldb multiples of 8 elements (TMA strides are
 * multiples of 16 bytes). D and ldd have no alignment rule (unaligned D takes a scalar
 * store path). M, N, K >= 0; K == 0 writes the epilogue of a zero accumulator.
 * Unlike the reference (K % 32 == 0, src/gemm_bench.cu:746) any K is accepted: the
 * ragged K tail is zero-filled by TMA.
 * ------------------------------------------------------------------------------------- */
int b2g_gemm(const void* A, const void* B, void* D, const void* bias, int M, int N, int K,
             long long lda, long long ldb, long long ldd, int b_layout, int acc, int epilogue,
             float alpha, int tile, int stages, int group, void* stream);

/* b2g_gemm with an explicit split-K factor. No counterpart in the reference, whose kernel
 * collapses on skinny shapes (docs/RESULTS.md:249-265: M = 1..128 with N = K = 4096 keep
 * 0.4-44% of its square-GEMM throughput) and names split-K as the fix.
 *   splits : 0 = automatic (what b2g_gemm does: split only when the output tiles fill less
 *            than half of the SMs, FP32 accumulation only), 1 = never, S >= 2 = split the
 *            K range of every tile into S even parts (S <= ceil(K / 64); acc must be
 *            B2G_ACC_F32, else B2G_ERR_UNSUPPORTED).
 * The partial sums of a tile's splits are added in split order 0..S-1 (deterministic, the
 * same bits on every call and through every entry point) before the epilogue. On the 1-CTA
 * tiles (128 x 64, 128 x 128, 128 x 256) with S <= 8, when the receive buffers fit in shared
 * memory (S <= 8 on 128 x 64 and 128 x 128, S = 2 on 128 x 256), the S splits of a tile run
 * as one thread-block cluster and each split stores its FP32 partials straight into the
 * shared memory of the CTA that sums them (distributed shared memory): no global workspace.
 * Otherwise (2-CTA tiles, larger S) each split writes its partial tile to a workspace and
 * the split that finishes last sums them. That workspace belongs to the library, one per
 * (device, stream), allocated with cudaMalloc on first use and grown when a larger one is
 * needed (after synchronising that stream). Growing is refused with B2G_ERR_UNSUPPORTED
 * while the stream is being captured, so run a call of each split shape once before
 * capturing it into a CUDA graph. B2G_SPLITK_CLUSTER=0 in the environment keeps every split
 * on the workspace path. */
int b2g_gemm_splitk(const void* A, const void* B, void* D, const void* bias, int M, int N,
                    int K, long long lda, long long ldb, long long ldd, int b_layout, int acc,
                    int epilogue, float alpha, int tile, int stages, int group, int splits,
                    void* stream);

/* b2g_gemm_splitk that allocates no device memory. No counterpart in the reference (which
 * has no split-K and no workspace). For callers that cannot allocate at call time: a
 * process whose free device memory is all held by its own caching allocator or a fixed
 * memory budget, or code where a cudaMalloc, a cudaFree or the stream synchronisation that
 * growing b2g_gemm_splitk's workspace needs is not acceptable.
 * Same arguments and results as b2g_gemm_splitk. The split-K scratch is a static device
 * array inside the library, one per device, of fixed size: 16 MiB of FP32 partials (a split
 * GEMM needs tiles x splits x 128 x 128 x 4 bytes on 128 x 128 tiles, x 2 x 2 on 2-CTA
 * 256 x 256 tiles) and 32768 counters (tiles x CTAs per tile x 8). A call needing more
 * returns B2G_ERR_ARG (with the sizes in the message) and launches nothing; calls that do
 * not split need no scratch. The counters must start at zero: they are zero-filled when the
 * library's module is loaded on the device and never need clearing later.
 * Limits: calls that can overlap on the same device (other streams, other host threads)
 * share the one array and race, so serialise them; make the first call on each device before
 * any stream capture, since it looks up the array's address (cudaGetSymbolAddress). The
 * address is kept for the life of the process: after a cudaDeviceReset (or any reset of the
 * device's primary context) the module is loaded again, maybe elsewhere, so no call of this
 * entry point, nor of b2g_gemm_splitk (whose workspace is cached the same way), may follow a
 * device reset in the same process. */
int b2g_gemm_splitk_noalloc(const void* A, const void* B, void* D, const void* bias, int M,
                            int N, int K, long long lda, long long ldb, long long ldd,
                            int b_layout, int acc, int epilogue, float alpha, int tile,
                            int stages, int group, int splits, void* stream);

/* One GEMM over `ngpu` devices by M-row panels, from one host process with one host thread
 * per device: the reference's multi-GPU plan (A split by rows, B replicated, no reduction;
 * the reference itself has no multi-GPU code). Device devices[g] computes rows
 * [M*g/ngpu, M*(g+1)/ngpu) of D. Per device, the caller passes pointers on that device:
 * A[g] = its panel of A (rows x K, lda), B[g] = a full copy of B, D[g] = its panel of D
 * (rows x N, ldd), bias[g] (bias may be NULL), streams[g] (streams may be NULL: the legacy
 * stream of each device). The other arguments mean what they mean for b2g_gemm. Returns
 * after every device's launch is enqueued, or with `sync` = 1 after every device finished
 * and its status word was checked (b2g_sync_status). A failure names the device. */
int b2g_gemm_multi(int ngpu, const int* devices, const void* const* A, const void* const* B,
                   void* const* D, const void* const* bias, int M, int N, int K, long long lda,
                   long long ldb, long long ldd, int b_layout, int acc, int epilogue, float alpha,
                   int tile, int stages, int group, void* const* streams, int sync);

/* All-gather of the D panels of b2g_gemm_multi over NVLink / NVSwitch: device g copies its
 * rows [M*g/ngpu, M*(g+1)/ngpu) (D[g], pitch ldd) into D_full[h] (M x N, pitch ldd, on device
 * h) for every h, with peer-to-peer copies on streams[g] (peer access is enabled as needed).
 * Each device's copies are ordered after its own earlier work on streams[g] only: for D_full
 * to be complete, synchronise every device's stream (or pass `sync` = 1). No counterpart in
 * the reference (its plan names an NCCL all-gather; this one needs no NCCL). */
int b2g_allgather_rows(int ngpu, const int* devices, void* const* D, void* const* D_full, int M,
                       int N, long long ldd, void* const* streams, int sync);

/* b2g_gemm_multi and the all-gather in one kernel per device: device g computes its rows
 * [M*g/ngpu, M*(g+1)/ngpu) from its A panel A[g] and a full copy of B, B[g], and its epilogue
 * writes every staged 32 x 64 box of the result both into its own D_full[g] (TMA stores) and,
 * with 16-byte stores over NVLink, into the same rows of every other device's D_full[h], so
 * the transfer overlaps the next tile's MMAs. D_full[g] is an M x N matrix (pitch ldd) on
 * device devices[g]. Needs 1 <= ngpu <= 8, peer access between every pair of devices, N % 8
 * == 0, ldd % 8 == 0 and 16-byte aligned D_full; tile 5 (swapped operands) is not offered.
 * With `sync` = 0 D_full[h] is complete once every device's stream has finished (kernel
 * completion makes the remote stores visible). No counterpart in the reference (its plan
 * names an NCCL all-gather after the GEMM). */
int b2g_gemm_multi_allgather(int ngpu, const int* devices, const void* const* A,
                             const void* const* B, void* const* D_full, const void* const* bias,
                             int M, int N, int K, long long lda, long long ldb, long long ldd,
                             int b_layout, int acc, int epilogue, float alpha, int tile,
                             int stages, int group, void* const* streams, int sync);

/* b2g_gemm on the current device whose epilogue also writes every element of D into each of
 * npeer (0..7) other copies of D: peer_D[i] addresses D's first row in a copy with the same
 * ldd, normally another device's memory (peer access enabled, or a CUDA IPC mapping from
 * b2g_ipc_open), reached with 16-byte stores over NVLink. The building block of the fused
 * all-gather for callers with one process per GPU: rank r passes its M-row panel of A and, as
 * D and peer_D, its rows in its own and every other rank's full D. Needs N % 8 == 0, ldd % 8
 * == 0 and 16-byte aligned D and copies; tile 5 is not offered. The copies are complete when
 * this launch has finished. No counterpart in the reference. */
int b2g_gemm_peers(const void* A, const void* B, void* D, const void* bias, int M, int N, int K,
                   long long lda, long long ldb, long long ldd, int b_layout, int acc,
                   int epilogue, float alpha, int tile, int stages, int group,
                   const void* const* peer_D, int npeer, void* stream);

/* CUDA IPC for the fused all-gather across processes. b2g_ipc_handle writes the 64-byte IPC
 * handle of the device allocation containing `ptr` and ptr's byte offset inside it;
 * another process maps that allocation with b2g_ipc_open (*base = its address there; add the
 * offset) and unmaps it with b2g_ipc_close(base). The allocation must come from cudaMalloc
 * (PyTorch's default caching allocator uses it); a process cannot open its own handles. */
int b2g_ipc_handle(const void* ptr, void* handle, unsigned long long* offset);
int b2g_ipc_open(const void* handle, void** base);
int b2g_ipc_close(void* base);

/* Message of the last failed call on this thread ("" if none). */
const char* b2g_last_error(void);

/* Synchronises `stream`, then reads and clears this device's status word. Returns
 * B2G_ERR_TIMEOUT if any kernel of this library gave up a bounded wait since the last
 * call (the message names the role and barrier), B2G_ERR_CUDA on a CUDA error. */
int b2g_sync_status(void* stream);

/* Clock telemetry of the most recent GEMM launch on the current device (call after the
 * launch completed, e.g. after b2g_sync_status): CTA 0 records globaltimer and clock64 at
 * entry and exit, so *sm_mhz = clock cycles / nanoseconds is the SM clock the kernel ran
 * at and *cta0_us the lifetime of CTA 0. No counterpart in the reference, which reads
 * clocks from nvidia-smi in its scripts (scripts/soak.ps1:38-62). */
int b2g_kernel_clock(double* sm_mhz, double* cta0_us);

/* Static properties of a configuration, for the report table columns the reference prints
 * from run_cfg (src/gemm_bench.cu:458-472): threads per CTA (the maximum, 320: a launch uses
 * 192 or 320, see b2g_last_launch), registers per thread, dynamic shared memory bytes,
 * resident CTAs per SM, TMEM columns, and the stage count used when `stages` is 0. Any
 * output pointer may be NULL. */
int b2g_config_info(int tile, int stages, int* threads, int* regs, int* smem_bytes,
                    int* ctas_per_sm, int* tmem_cols, int* stages_used);

/* The most recent GEMM kernel launch made by b2g_gemm / b2g_gemm_splitk on the calling host
 * thread: grid size, threads per CTA (64 + 32 x epilogue warps: 8 epilogue warps when
 * K <= 1024, else 4), the tile and stage count chosen, the work units (tiles x splits, plus
 * tail slices) and the split-K factor. The reference prints the same launch facts per
 * configuration (src/gemm_bench.cu:458-472); here they depend on the shape, so they are read
 * back after the call. Any output pointer may be NULL; B2G_ERR_ARG if this thread has not
 * launched a GEMM yet. */
int b2g_last_launch(int* grid, int* threads, int* tile, int* stages, int* units, int* splits);

/* Thread-block cluster size of the same most recent launch: 1 for the 1-CTA kernels, 2 for
 * the 2-CTA pair kernels, and S for a 1-CTA split-K launch whose S splits of each tile form
 * one cluster and are summed through distributed shared memory. No counterpart in the
 * reference (its kernel uses no clusters). B2G_ERR_ARG before any launch on this thread. */
int b2g_last_launch_cluster(int* cluster_ctas);

/* Which compiled form of the tile kernel the same most recent launch ran:
 * B2G_VARIANT_GENERAL (every mode a runtime branch: FP16 accumulation, fused epilogue,
 * workspace split-K, K x N B on the pair kernel; also the swapped-operand kernel),
 * B2G_VARIANT_PEERS (the fused all-gather of b2g_gemm_peers), B2G_VARIANT_PLAIN (no split-K,
 * FP32 accumulation, plain store, no peers, compiled as constants) or B2G_VARIANT_CSPLIT
 * (split-K summed in a cluster, FP32 accumulation, no peers), or B2G_VARIANT_NARROW (the
 * swapped-operand kernel's narrow form: ~N / SMs rows of B per CTA over the whole K range,
 * chosen when its 128-row blocks would leave more than half of the SMs idle). The choice follows from the
 * arguments; the results do not depend on it. No counterpart in the reference (one kernel).
 * B2G_ERR_ARG before any launch on this thread. */
#define B2G_VARIANT_GENERAL 0
#define B2G_VARIANT_PEERS 1
#define B2G_VARIANT_PLAIN 2
#define B2G_VARIANT_CSPLIT 3
#define B2G_VARIANT_NARROW 4
int b2g_last_launch_variant(int* variant);

/* cuBLAS comparison column: exactly the reference's call (src/gemm_bench.cu:625-633):
 * cublasGemmEx(OP_T, OP_N, N, M, K, alpha, B, 16F, K, A, 16F, K, beta=0, D, 16F, N,
 * COMPUTE_32F, DEFAULT_TENSOR_OP) on `stream`, with tensor-op math mode
 * (src/gemm_bench.cu:777-778). Uses one cached handle per thread and device. */
int b2g_cublas_gemm(const void* A, const void* B, void* D, int M, int N, int K, void* stream);

/* Device-side max |x - y| / max(1, |y|) over n FP16 values into *out_dev (FP32, device
 * memory). Replaces max_rel_diff (src/gemm_bench.cu:648-664). */
int b2g_max_rel_diff(const void* x, const void* y, size_t n, float* out_dev, void* stream);

/* Unfused epilogue: D = relu(alpha * D + bias[n]) in place (bias may be NULL). Replaces
 * bias_relu_kernel (src/gemm_bench.cu:401-408), the reference's --unfused comparison. */
int b2g_bias_relu(void* D, const void* bias, int M, int N, long long ldd, float alpha,
                  void* stream);

/* tcgen05 issue-rate probe. Replaces mma_probe / probe_one / probe
 * (src/device_query.cu:48-163, 199-224), which time register-resident mma.sync.
 *   kind     : 0 kind::f16 F16 in, F32 accumulate   1 kind::f16 F16 in, F16 accumulate
 *              2 kind::i8 S8 in, S32 accumulate      3 kind::f8f6f4 E4M3 in, F32 accumulate
 *   cta_group: 1 = one CTA per SM issuing UMMA M = 128 (the 1-CTA GEMM kernels);
 *              2 = 2-CTA clusters, the even CTA issuing the pair MMA (UMMA M = 256 over two
 *              SMs, each holding half of A, half of B and its 128 accumulator lanes), as the
 *              2-CTA GEMM kernels do
 *   n        : UMMA N, 16..256 in steps of 16
 *   iters    : back-to-back MMAs per CTA or pair (operands resident in shared memory,
 *              accumulator in TMEM, no memory traffic in the loop)
 * One CTA per SM (cta_group 1) or one cluster per two SMs (cta_group 2); clock64-timed on
 * the device like the reference. Outputs the best (fewest-cycle) CTA's or pair's dense FLOP
 * per clock per SM (a pair's FLOP divided over its two SMs) and its cycles. */
int b2g_probe_tcgen05(int kind, int cta_group, int n, int iters, double* flop_per_clk_sm,
                      long long* cycles);

/* HBM stream probe: `reps` copies of `bytes` from src to dst (both device, caller-owned,
 * 16-byte aligned), timed with CUDA events on `stream`. Replaces bw_kernel /
 * probe_bandwidth (src/device_query.cu:165-197). Outputs read+write GB/s. */
int b2g_probe_hbm(const void* src, void* dst, size_t bytes, int reps, void* stream,
                  double* gbs);

/* Host input generators (the same values on every machine).
 * b2g_fill_lcg_f16 reproduces the reference's deterministic init bit for bit
 * (src/gemm_bench.cu:760-765): A, then B (N x K order), then bias.
 * b2g_fill_uniform_f16 is the seeded counter-based generator of the synthetic inputs;
 * dst[j] gets the value of global element index i = first + j (so a row panel of a
 * larger matrix can be generated on its own):
 *   key = mix(seed * 0x9E3779B97F4A7C15 ^ (tensor_id + 1) * 0xD1B54A32D192ED03)
 *   u   = (mix(key + i * 0x9E3779B97F4A7C15) >> 40) * 2^-24,  v = lo + (hi - lo) * u
 * (mix = the splitmix64 finaliser), rounded to FP16 (RNE). Multi-threaded. */
void b2g_fill_lcg_f16(uint16_t* A, long long nA, uint16_t* B, long long nB, uint16_t* bias,
                      long long nbias);
void b2g_fill_uniform_f16(uint16_t* dst, long long n, long long first, uint64_t seed,
                          uint32_t tensor_id, double lo, double hi);

/* Tile scheduler mapping used by every persistent GEMM kernel: linear tile id ->
 * (m_tile, n_tile). Same rasterization as src/gemm_bench.cu:237-250. */
void b2g_tile_coord(int linear, int tiles_m, int tiles_n, int group, int* m_tile,
                    int* n_tile);

/* Failure-detection self-test: launches one CTA that waits on an mbarrier nothing
 * arrives at, with a wait limit of `timeout_us` microseconds (1..2,000,000). The wait
 * gives up, records B2G_ERR_TIMEOUT in the status word and the kernel returns; the call
 * then returns what b2g_sync_status() returns (B2G_ERR_TIMEOUT when working). The CUDA
 * context stays usable. No counterpart in the reference (it has fail-fast exit() only,
 * src/gemm_bench.cu:59-76). */
int b2g_selftest_wait_timeout(unsigned timeout_us, void* stream);

/* Device-side wait limit used by every kernel of this library, in microseconds
 * (default 4,000,000; the environment variable B2G_WAIT_TIMEOUT_US overrides it).
 * Returns the previous value. */
unsigned long long b2g_set_wait_timeout_us(unsigned long long us);

/* Library version (major*10000 + minor*100 + patch). */
int b2g_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B2G_H */
