// sm100_ptx.cuh -- inline-PTX primitives for sm_100a: mbarriers, TMA tile loads, tensor
// memory (TMEM) allocation, tcgen05.mma / commit / ld, and the shared-memory and
// instruction descriptors that tcgen05.mma consumes.
//
// These replace the reference's sm_80 primitives (src/gemm_bench.cu:78-152: cp.async,
// ldmatrix, mma.sync). Every wait on an mbarrier is bounded: it gives up after a time
// limit, records the failure in the device status word and tells the caller to unwind.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace b2g {

// Bits of the device status word (read and cleared by b2g_sync_status).
enum : uint32_t {
    kErrWaitProducer = 1u << 0,  // TMA producer gave up waiting for a free stage
    kErrWaitMma = 1u << 1,       // MMA issuer gave up waiting for a full stage / free TMEM
    kErrWaitEpilogue = 1u << 2,  // epilogue gave up waiting for a finished accumulator
    kErrWaitSelftest = 1u << 3,  // the self-test's deliberately unsatisfied wait
    kErrWaitDrain = 1u << 4,     // teardown gave up waiting for in-flight async work
    kErrWaitProbe = 1u << 5,     // issue-rate probe gave up waiting for its MMAs
    kErrSplitCounter = 1u << 6   // a split-K arrival counter update did not go through
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// ---------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on an mbarrier of another CTA in the cluster (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
                 : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok;
}

// Cluster-scope acquire: for barriers that a peer CTA's operations complete.
__device__ __forceinline__ uint32_t mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok;
}

// Map a shared::cta address of this CTA to the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
    return out;
}

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
    cluster_arrive();
    cluster_wait();
}

// Bounded-wait context: a time limit, the CTA's abort flag (shared memory) and the status
// bit this role sets when it gives up.
struct WaitCtx {
    unsigned long long limit_ns;
    volatile int* abort_flag;
    uint32_t err_bit;
};

__device__ unsigned int g_b2g_status;  // per-device status word, see b2g_sync_status()

__device__ __forceinline__ void raise_status(uint32_t bits) {
    atomicOr(&g_b2g_status, bits);
}

// Clock telemetry of the last GEMM launch, written by CTA 0 of the grid:
// [0] globaltimer at start (ns), [1] at exit, [2] clock64 at start, [3] at exit.
// (clock64 delta / globaltimer delta = the SM clock the kernel actually ran at.)
__device__ unsigned long long g_b2g_clock[4];

__device__ __forceinline__ void clock_mark(int at_exit) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        g_b2g_clock[at_exit] = globaltimer_ns();
        g_b2g_clock[2 + at_exit] = (unsigned long long)clock64();
    }
}

// Optional wait-time instrumentation (build with -DB2G_INSTRUMENT; off in the library):
// per CTA, clock64 cycles each role spent inside its barrier waits, plus the CTA's
// lifetime. Slots: 0 producer/empty, 1 MMA/full, 2 MMA/tmem_empty, 3 epilogue/tmem_full
// (warp 2), 4 epilogue work (warp 2), 5 CTA lifetime, 6 k-blocks issued, 7 units;
// epilogue chunk phases of thread 64 (warp 2, lane 0): 8 TMEM load + wait, 9 convert +
// shared stores, 10 wait for the staging box, 11 fence + store issue, 12 chunks; split-K
// units instead: 12 reduction cycles, 13 partial store + release, 14 arrival, 15 reductions.
#ifdef B2G_INSTRUMENT
constexpr int kInstrSlots = 16;
__device__ unsigned long long g_b2g_instr[1024][kInstrSlots];
#define B2G_TIC(v) const long long v = clock64()
#define B2G_TOC(slot, v) \
    atomicAdd(&g_b2g_instr[blockIdx.x][slot], (unsigned long long)(clock64() - (v)))
#define B2G_COUNT(slot, n) atomicAdd(&g_b2g_instr[blockIdx.x][slot], (unsigned long long)(n))
#define B2G_TOC64(slot, v) \
    if (threadIdx.x == 64) B2G_TOC(slot, v)
// Timeline of every CTA (globaltimer ns, [CTA][mark]): mark i is written by whichever thread
// of the CTA reaches it. 1-CTA kernel: 0 entry, 1 barriers and TMEM ready (cluster synced),
// 2 after griddepcontrol.wait, 3 first TMA load issued, 4 first stage full at the MMA warp,
// 5 accumulator committed, 6-9 cluster split-K epilogue of thread 128 (start, sends issued,
// receive wait done, end), 10 after the teardown barriers, 11 producer issued its last load,
// 12-14 epilogue thread 64: first accumulator ready, last unit's epilogue done, stores read.
// 15 producer's first empty wait done; 16-18 epilogue thread 64, first chunk: TMEM load
// done, first half staged, store issued. Slots 24 + i hold clock64() at mark i.
constexpr int kTlMarks = 24;
__device__ unsigned long long g_b2g_tl[1024][2 * kTlMarks];
#define B2G_MARK(i)                                                    \
    if (blockIdx.x < 1024) {                                           \
        g_b2g_tl[blockIdx.x][kTlMarks + (i)] = (unsigned long long)clock64(); \
        g_b2g_tl[blockIdx.x][i] = globaltimer_ns();                    \
    }
#else
#define B2G_MARK(i)
#define B2G_TOC64(slot, v)
#define B2G_TIC(v)
#define B2G_TOC(slot, v)
#define B2G_COUNT(slot, n)
#endif

// Waits until the phase with parity `parity` of `bar` has completed. Returns false if the
// CTA is aborting or the time limit ran out (then it sets the status bit and the abort
// flag so the other roles unwind too). CLUSTER selects cluster-scope acquire.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w) {
    if (CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
        if (CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity))
            return true;
        if ((++spins & 15u) == 0u) {
            if (*w.abort_flag) return false;
            if (globaltimer_ns() - t0 > w.limit_ns) {
                raise_status(w.err_bit);
                *w.abort_flag = 1;
                return false;
            }
        }
    }
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization
// may start while the previous kernel in the stream is still running; `grid_dep_wait`
// blocks until that kernel has completed and its memory is visible (every thread calls it
// before its first global-memory access), and `grid_dep_launch` lets the next kernel start
// its own prologue on SMs this grid frees.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One lane of the (converged) warp gets true. Role loops run on whole warps and issue their
// single-thread instructions (tcgen05.mma / commit, TMA) from the elected lane, so their
// operands stay warp-uniform (uniform datapath) instead of being rebuilt per issue.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// Bounded wait by a whole warp: every lane polls, the warp agrees on the outcome.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, const WaitCtx& w) {
    const bool ok = mbar_wait<CLUSTER>(bar, parity, w);
    return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) -- plain tile loads, no multicast anywhere in this library.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// 2D tile load into this CTA's shared memory; completion counted on `bar` (this CTA).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// 2D tile load into this CTA's shared memory whose completion is signalled on an mbarrier
// that may live in the peer CTA of a 2-CTA pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* tm,
                                                 uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// 3D tile loads (same completion forms as the 2D ones above): used for B stored K x N, whose
// 64-column groups are the outer dimension of the tensor map, so one load brings a CTA's
// whole stage of B (several 64-column x 64-k-row boxes, back to back) instead of one load
// per 64-column box.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* tm,
                                                 uint32_t bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ unsigned short ld_shared_u16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
    return v;
}

// 16-byte store into the shared memory of another CTA of the cluster (`addr` from
// mapa_shared) whose bytes are counted on that CTA's mbarrier `bar` (also a mapa address):
// the receiver arms the barrier with the bytes it expects and waits on it, as for a TMA load.
__device__ __forceinline__ void st_async_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                            uint32_t d, uint32_t bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, "
        "[%5];" ::"r"(addr),
        "r"(a), "r"(b), "r"(c), "r"(d), "r"(bar)
        : "memory");
}

// gpu-scope relaxed load and acquire-release compare-and-swap (split-K arrival counters).
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long atom_cas_acq_rel_gpu_u64(unsigned long long* p,
                                                                       unsigned long long cmp,
                                                                       unsigned long long val) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.cas.b64 %0, [%1], %2, %3;"
                 : "=l"(old)
                 : "l"(p), "l"(cmp), "l"(val)
                 : "memory");
    return old;
}

// L2 cache policies (createpolicy) for the `.L2::cache_hint` forms below.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* tm,
                                                 uint32_t bar, int c0, int c1, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t dst, const CUtensorMap* tm,
                                                      uint32_t bar, int c0, int c1,
                                                      uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "l"(pol)
        : "memory");
}

// 2D tile store with an L2 cache policy (e.g. evict_first for output that is not re-read).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* tm, uint32_t src, int c0,
                                                  int c1, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint"
        " [%0, {%2, %3}], [%1], %4;" ::"l"(reinterpret_cast<uint64_t>(tm)),
        "r"(src), "r"(c0), "r"(c1), "l"(pol)
        : "memory");
}

// 2D tile store from this CTA's shared memory (bulk async-group completion). The tensor map
// clips rows / columns outside the tensor; callers never start a store at a negative
// coordinate.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, uint32_t src, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(tm)),
        "r"(src), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// at most N of this thread's bulk groups may still be reading their shared memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// at most N of this thread's bulk groups may still be in flight at all
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// 16-byte store with the streaming (evict-first) hint; `ptr` may be a peer device's memory
// (peer access enabled), in which case the store crosses NVLink.
__device__ __forceinline__ void st_global_cs_v4(void* ptr, uint4 v) {
    asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---------------------------------------------------------------------------------------
// Tensor memory and tcgen05
// ---------------------------------------------------------------------------------------
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         dst_smem),
                     "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         dst_smem),
                     "r"(ncols)
                     : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
    if constexpr (CG == 1)
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    else
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
                     "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr),
                     "r"(ncols)
                     : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy
// (TMA, tensor core) before they are consumed there.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (F16 or BF16 inputs).
template <int CG>
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
    if constexpr (CG == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// kind::i8 (S8 x S8 -> S32) and kind::f8f6f4 (here E4M3 x E4M3 -> F32), cta_group::1 or ::2.
template <int CG = 1>
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    if constexpr (CG == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
}
template <int CG = 1>
__device__ __forceinline__ void mma_f8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    if constexpr (CG == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// Arrive (once) on `bar` when all tcgen05 operations this thread issued so far complete.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// 2-CTA form (all tcgen05 ops of a kernel use one cta_group): arrive on this CTA's `bar`.
__device__ __forceinline__ void mma_commit_2(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// 2-CTA form: arrive on the barrier at offset `bar` in every CTA of `cta_mask`.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(bar),
        "h"(cta_mask)
        : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: lane i of the warp gets TMEM lane
// (taddr.lane + i), register j holds column (taddr.col + j).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// 64 consecutive columns: two 32-column loads into one 64-register array.
__device__ __forceinline__ void tmem_ld_32x32b_x64(uint32_t taddr, uint32_t (&r)[64]) {
    tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
    tmem_ld_32x32b_x32(taddr + 32u, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 format): start address, leading- and
// stride-dimension byte offsets (all >> 4), version 1 at bit 46, swizzle mode at 61..63
// (2 = 128-byte swizzle). Operand tiles are 1024-byte aligned so the base offset is 0.
//
// K-major operand written by TMA with SWIZZLE_128B and a 64-element (128 B) inner box:
// row r of the tile sits at r * 128 B, 8-row groups (1024 B swizzle atoms) follow at
// SBO = 1024 B; LBO is unused for swizzled K-major layouts. The k-th 16-element step of
// one MMA starts 32 * k bytes into the row.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::f16: dense, F16 A and B, D = F32 (acc_f32) or F16,
// A K-major, B K-major (b_mn_major = 0) or MN-major (1), N >> 3 at bits 17..22,
// M >> 4 at bits 24..28.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool acc_f32, bool b_mn_major) {
    return ((acc_f32 ? 1u : 0u) << 4) | (0u << 7) | (0u << 10) | (0u << 15) |
           ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

}  // namespace b2g
