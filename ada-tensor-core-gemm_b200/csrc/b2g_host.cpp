// b2g_host.cpp -- host-only part of libb200gemm.so: error reporting, device facts, the
// cuBLAS comparison column, the host input generators, the tile-scheduler mapping, the
// multi-GPU entry points and CUDA IPC sharing of D buffers between processes.
#include <cublas_v2.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <omp.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "b2g.h"
#include "b2g_internal.h"
#include "tile_sched.h"

namespace b2g {

namespace {
thread_local std::string t_last_error;
std::mutex g_mu;
unsigned long long g_timeout_us = 0;  // 0 = not initialised yet
DeviceInfo g_dev[64];
}  // namespace

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

void clear_error() { t_last_error.clear(); }

unsigned long long wait_timeout_ns() {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_timeout_us == 0) {
        g_timeout_us = 4000000ull;
        if (const char* e = std::getenv("B2G_WAIT_TIMEOUT_US")) {
            const unsigned long long v = std::strtoull(e, nullptr, 10);
            if (v > 0) g_timeout_us = v;
        }
    }
    return g_timeout_us * 1000ull;
}

int current_device(DeviceInfo& out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0)
        return fail(B2G_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
    if (dev < 64) {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_dev[dev].device == dev) {
            out = g_dev[dev];
            return B2G_OK;
        }
    }
    DeviceInfo di;
    di.device = dev;
    cudaDeviceGetAttribute(&di.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&di.minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&di.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&di.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (di.major != 10 || di.minor != 0)
        return fail(B2G_ERR_NO_DEVICE,
                    "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev,
                    di.major, di.minor);
    if (dev < 64) {
        std::lock_guard<std::mutex> lock(g_mu);
        g_dev[dev] = di;
    }
    out = di;
    return B2G_OK;
}

namespace {

uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// IEEE binary32 -> binary16, round to nearest even (what __float2half does on the host).
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (ax >= 0x38800000u) {
        uint32_t h = ((((ax >> 23) - 112u) << 10) | ((ax & 0x7FFFFFu) >> 13));
        const uint32_t rem = ax & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    const uint32_t e = ax >> 23;
    if (e == 0) return (uint16_t)sign;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const int shift = 126 - (int)e;
    if (shift >= 32) return (uint16_t)sign;
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

struct CublasSlot {
    int device = -1;
    cublasHandle_t h = nullptr;
};
thread_local CublasSlot t_cublas[64];

}  // namespace
}  // namespace b2g

using namespace b2g;

B2G_EXPORT const char* b2g_last_error(void) { return t_last_error.c_str(); }

B2G_EXPORT unsigned long long b2g_set_wait_timeout_us(unsigned long long us) {
    const unsigned long long prev = wait_timeout_ns() / 1000ull;
    if (us > 0) {
        std::lock_guard<std::mutex> lock(g_mu);
        g_timeout_us = us;
    }
    return prev;
}

B2G_EXPORT int b2g_version(void) { return 100; }  // 0.1.0

B2G_EXPORT void b2g_tile_coord(int linear, int tiles_m, int tiles_n, int group, int* m_tile,
                               int* n_tile) {
    int m = 0, n = 0;
    tile_coord(linear, tiles_m, tiles_n, group, m, n);
    if (m_tile) *m_tile = m;
    if (n_tile) *n_tile = n;
}

// The reference's init (src/gemm_bench.cu:760-765), bit for bit.
B2G_EXPORT void b2g_fill_lcg_f16(uint16_t* A, long long nA, uint16_t* B, long long nB,
                                 uint16_t* bias, long long nbias) {
    uint32_t s = 12345u;
    auto rnd = [&] {
        s = s * 1664525u + 1013904223u;
        return (float)((s >> 16) & 1023u) / 1023.f - 0.5f;
    };
    for (long long i = 0; i < nA; ++i) A[i] = f32_to_f16(rnd());
    for (long long i = 0; i < nB; ++i) B[i] = f32_to_f16(rnd());
    for (long long i = 0; i < nbias; ++i) bias[i] = f32_to_f16(rnd());
}

B2G_EXPORT void b2g_fill_uniform_f16(uint16_t* dst, long long n, long long first,
                                     uint64_t seed, uint32_t tensor_id, double lo, double hi) {
    const uint64_t key =
        mix64(seed * 0x9E3779B97F4A7C15ull ^ ((uint64_t)tensor_id + 1ull) * 0xD1B54A32D192ED03ull);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < n; ++i) {
        const uint64_t h = mix64(key + (uint64_t)(first + i) * 0x9E3779B97F4A7C15ull);
        const double u = (double)(h >> 40) * (1.0 / 16777216.0);
        const double v = lo + (hi - lo) * u;
        dst[i] = f32_to_f16((float)v);
    }
}

// The reference's cuBLAS speed-of-light call (src/gemm_bench.cu:621-633): row-major
// D(M x N) = A(M x K) * B(N x K)^T computed as column-major D^T = B^T * A^T.
B2G_EXPORT int b2g_cublas_gemm(const void* A, const void* B, void* D, int M, int N, int K,
                               void* stream) {
    clear_error();
    if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_ARG, "negative shape");
    if (M == 0 || N == 0) return B2G_OK;
    DeviceInfo di;
    if (int rc = current_device(di)) return rc;
    CublasSlot& slot = t_cublas[di.device & 63];
    if (slot.device != di.device || !slot.h) {
        cublasHandle_t h = nullptr;
        if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS)
            return fail(B2G_ERR_LIBRARY, "cublasCreate failed");
        cublasSetMathMode(h, CUBLAS_TENSOR_OP_MATH);
        slot.device = di.device;
        slot.h = h;
    }
    cublasSetStream(slot.h, (cudaStream_t)stream);
    const float alpha = 1.f, beta = 0.f;
    cublasStatus_t st = cublasGemmEx(slot.h, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &alpha, B,
                                      CUDA_R_16F, K, A, CUDA_R_16F, K, &beta, D, CUDA_R_16F, N,
                                      CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT_TENSOR_OP);
    if (st != CUBLAS_STATUS_SUCCESS) return fail(B2G_ERR_LIBRARY, "cublasGemmEx: status %d", (int)st);
    return B2G_OK;
}

// ---------------------------------------------------------------------------------------
// Multi-GPU: M-row panels from one process (the reference's multi-GPU plan; it has no
// multi-GPU code of its own). One persistent host thread per device.
// ---------------------------------------------------------------------------------------
#include <pthread.h>

#include <atomic>
#include <condition_variable>
#include <deque>
#include <functional>
#include <memory>
#include <thread>
#include <vector>

namespace b2g {
namespace {

// Rows [r0, r1) of panel g of ngpu: M split as evenly as possible.
inline void panel_rows(int M, int ngpu, int g, int& r0, int& r1) {
    r0 = (int)((long long)M * g / ngpu);
    r1 = (int)((long long)M * (g + 1) / ngpu);
}

// One persistent host thread per device ordinal, started on first use. A call hands each of
// its devices' workers a task and waits for all of them: spawning a thread per device per
// call measured ~250 us for 8 devices on an 8-core host (more than an 8192^3 GEMM's share of
// one GPU), a hand-off to a waiting thread a few us. Tasks for one device (a device listed
// twice) run one after the other on its worker. The pool is never destroyed (idle workers end
// with the process); a forked child starts a fresh, empty pool. A task must not wait for
// another task.
class DeviceWorkers {
  public:
    static DeviceWorkers& get() {
        static const bool hooked = [] {
            pthread_atfork(nullptr, nullptr, [] { current().store(new DeviceWorkers()); });
            return true;
        }();
        (void)hooked;
        DeviceWorkers* w = current().load();
        if (!w) {
            DeviceWorkers* fresh = new DeviceWorkers();
            if (current().compare_exchange_strong(w, fresh)) return *fresh;
            delete fresh;  // another thread installed one first
        }
        return *w;
    }

    // Queues `task` on the worker of `device`; false if the worker thread could not start.
    bool post(int device, std::function<void()> task) {
        Worker* w = worker(device);
        if (!w) return false;
        {
            std::lock_guard<std::mutex> lock(w->mu);
            w->q.push_back(std::move(task));
        }
        w->cv.notify_one();
        return true;
    }

  private:
    struct Worker {
        std::mutex mu;
        std::condition_variable cv;
        std::deque<std::function<void()>> q;
    };

    static std::atomic<DeviceWorkers*>& current() {
        static std::atomic<DeviceWorkers*> p{nullptr};
        return p;
    }

    Worker* worker(int device) {
        std::lock_guard<std::mutex> lock(mu_);
        if ((int)workers_.size() <= device) workers_.resize((size_t)device + 1);
        if (!workers_[(size_t)device]) {
            std::unique_ptr<Worker> w(new Worker());
            try {
                std::thread([p = w.get()] { loop(p); }).detach();
            } catch (...) {
                return nullptr;
            }
            workers_[(size_t)device] = std::move(w);
        }
        return workers_[(size_t)device].get();
    }

    static void loop(Worker* w) {
        for (;;) {
            std::function<void()> task;
            {
                std::unique_lock<std::mutex> lock(w->mu);
                w->cv.wait(lock, [w] { return !w->q.empty(); });
                task = std::move(w->q.front());
                w->q.pop_front();
            }
            task();
        }
    }

    std::mutex mu_;
    std::vector<std::unique_ptr<Worker>> workers_;  // by device ordinal; Workers never move
};

// Every listed device must be a visible CUDA device.
int check_devices(int ngpu, const int* devices) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return fail(B2G_ERR_NO_DEVICE, "no CUDA device: %s",
                    e != cudaSuccess ? cudaGetErrorString(e) : "count is 0");
    }
    for (int g = 0; g < ngpu; ++g)
        if (devices[g] < 0 || devices[g] >= n)
            return fail(B2G_ERR_ARG, "devices[%d] = %d: %d device(s) visible", g, devices[g], n);
    return B2G_OK;
}

// True if every pair of distinct listed devices has direct peer access (NVLink / NVSwitch).
bool all_peers_reachable(int ngpu, const int* devices) {
    for (int g = 0; g < ngpu; ++g)
        for (int h = 0; h < ngpu; ++h) {
            if (devices[h] == devices[g]) continue;
            int ok = 0;
            if (cudaDeviceCanAccessPeer(&ok, devices[g], devices[h]) != cudaSuccess || !ok)
                return false;
        }
    return true;
}

// On the current device (a worker's): enable direct access to every other listed device that
// it can reach. Asked on every call rather than remembered, so that access the application
// disabled in between is back before a kernel stores into a peer (an already-enabled pair
// costs one quick runtime call).
int enable_peers_from(int self, int ngpu, const int* devices) {
    for (int h = 0; h < ngpu; ++h) {
        const int peer = devices[h];
        if (peer == self) continue;
        int ok = 0;
        if (cudaDeviceCanAccessPeer(&ok, self, peer) != cudaSuccess || !ok) continue;
        cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
        if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
            return fail(B2G_ERR_CUDA, "peer access %d -> %d: %s", self, peer, cudaGetErrorString(e));
        cudaGetLastError();  // clears cudaErrorPeerAccessAlreadyEnabled
    }
    return B2G_OK;
}

// Runs fn(g) for every listed device on that device's worker (device current) and waits for
// all of them; the first failure (in list order) becomes the caller's error, naming the device.
// The caller's own current device is left as it was.
template <class Fn>
int for_each_device(int ngpu, const int* devices, Fn fn) {
    if (int rc = check_devices(ngpu, devices)) return rc;
    std::vector<int> rc((size_t)ngpu, B2G_OK);
    std::vector<std::string> msg((size_t)ngpu);
    std::mutex mu;
    std::condition_variable cv;
    int left = ngpu;
    auto done = [&] {
        std::lock_guard<std::mutex> lock(mu);
        if (--left == 0) cv.notify_all();
    };
    for (int g = 0; g < ngpu; ++g) {
        const bool posted = DeviceWorkers::get().post(devices[g], [&, g] {
            cudaError_t e = cudaSetDevice(devices[g]);
            if (e != cudaSuccess) {
                rc[(size_t)g] = B2G_ERR_CUDA;
                msg[(size_t)g] = std::string("cudaSetDevice: ") + cudaGetErrorString(e);
            } else {
                rc[(size_t)g] = fn(g);
                if (rc[(size_t)g] != B2G_OK) msg[(size_t)g] = b2g_last_error();
            }
            done();
        });
        if (!posted) {
            rc[(size_t)g] = B2G_ERR_CUDA;
            msg[(size_t)g] = "could not start the device's host worker thread";
            done();
        }
    }
    {
        std::unique_lock<std::mutex> lock(mu);
        cv.wait(lock, [&] { return left == 0; });
    }
    for (int g = 0; g < ngpu; ++g)
        if (rc[(size_t)g] != B2G_OK)
            return b2g::fail(rc[(size_t)g], "device %d (panel %d of %d): %s", devices[g], g, ngpu,
                             msg[(size_t)g].c_str());
    return B2G_OK;
}

}  // namespace
}  // namespace b2g

B2G_EXPORT int b2g_gemm_multi(int ngpu, const int* devices, const void* const* A,
                              const void* const* B, void* const* D, const void* const* bias,
                              int M, int N, int K, long long lda, long long ldb, long long ldd,
                              int b_layout, int acc, int epilogue, float alpha, int tile,
                              int stages, int group, void* const* streams, int sync) {
    using namespace b2g;
    clear_error();
    if (ngpu < 1 || !devices || !A || !B || !D)
        return fail(B2G_ERR_ARG, "ngpu >= 1 and the devices, A, B, D arrays are required");
    if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_ARG, "negative shape M=%d N=%d K=%d", M, N, K);
    return for_each_device(ngpu, devices, [&](int g) -> int {
        int r0, r1;
        panel_rows(M, ngpu, g, r0, r1);
        void* s = streams ? streams[g] : nullptr;
        int rc = b2g_gemm(A[g], B[g], D[g], bias ? bias[g] : nullptr, r1 - r0, N, K, lda, ldb,
                          ldd, b_layout, acc, epilogue, alpha, tile, stages, group, s);
        if (rc == B2G_OK && sync) rc = b2g_sync_status(s);
        return rc;
    });
}

B2G_EXPORT int b2g_allgather_rows(int ngpu, const int* devices, void* const* D,
                                  void* const* D_full, int M, int N, long long ldd,
                                  void* const* streams, int sync) {
    using namespace b2g;
    clear_error();
    if (ngpu < 1 || !devices || !D || !D_full)
        return fail(B2G_ERR_ARG, "ngpu >= 1 and the devices, D, D_full arrays are required");
    if (M < 0 || N < 0 || ldd < N) return fail(B2G_ERR_ARG, "bad shape M=%d N=%d ldd=%lld", M, N, ldd);
    // SM-driven push (one HBM read, ngpu stores of every 16 bytes) when the rows are 16-byte
    // groups and every pair of devices has peer access; else copy-engine 2D copies.
    if (int rc = check_devices(ngpu, devices)) return rc;
    bool push = ngpu <= kMaxGatherDst && N % 8 == 0 && ldd % 8 == 0 &&
                all_peers_reachable(ngpu, devices);
    for (int g = 0; g < ngpu && push; ++g)
        push = !(((uintptr_t)D[g] | (uintptr_t)D_full[g]) & 15);
    return for_each_device(ngpu, devices, [&](int g) -> int {
        if (int rc = enable_peers_from(devices[g], ngpu, devices)) return rc;
        int r0, r1;
        panel_rows(M, ngpu, g, r0, r1);
        cudaStream_t s = streams ? (cudaStream_t)streams[g] : nullptr;
        const size_t pitch = (size_t)ldd * 2;
        if (push) {
            void* dst[kMaxGatherDst];
            for (int k = 0; k < ngpu; ++k)  // start at a different peer on every device
                dst[k] = static_cast<char*>(D_full[(g + k) % ngpu]) + (size_t)r0 * pitch;
            if (int rc = allgather_push(D[g], r1 - r0, N, ldd, dst, ngpu, s)) return rc;
        } else {
            for (int k = 0; k < ngpu && r1 > r0; ++k) {
                const int h = (g + k) % ngpu;
                cudaError_t e = cudaMemcpy2DAsync(static_cast<char*>(D_full[h]) + (size_t)r0 * pitch,
                                                  pitch, D[g], pitch, (size_t)N * 2,
                                                  (size_t)(r1 - r0), cudaMemcpyDefault, s);
                if (e != cudaSuccess)
                    return fail(B2G_ERR_CUDA, "panel copy to device %d: %s", devices[h],
                                cudaGetErrorString(e));
            }
        }
        if (sync) {
            cudaError_t e = cudaStreamSynchronize(s);
            if (e != cudaSuccess)
                return fail(B2G_ERR_CUDA, "all-gather synchronize: %s", cudaGetErrorString(e));
        }
        return B2G_OK;
    });
}

B2G_EXPORT int b2g_gemm_multi_allgather(int ngpu, const int* devices, const void* const* A,
                                        const void* const* B, void* const* D_full,
                                        const void* const* bias, int M, int N, int K,
                                        long long lda, long long ldb, long long ldd, int b_layout,
                                        int acc, int epilogue, float alpha, int tile, int stages,
                                        int group, void* const* streams, int sync) {
    using namespace b2g;
    clear_error();
    if (ngpu < 1 || ngpu > kMaxPeerDst + 1 || !devices || !A || !B || !D_full)
        return fail(B2G_ERR_ARG, "ngpu in 1..%d and the devices, A, B, D_full arrays are required",
                    kMaxPeerDst + 1);
    if (M < 0 || N < 0 || K < 0) return fail(B2G_ERR_ARG, "negative shape M=%d N=%d K=%d", M, N, K);
    if (ldd < N) return fail(B2G_ERR_ARG, "ldd (%lld) < N (%d)", ldd, N);
    for (int g = 0; g < ngpu; ++g)
        if (!D_full[g]) return fail(B2G_ERR_ARG, "D_full[%d] is NULL", g);
    if (int rc = check_devices(ngpu, devices)) return rc;
    if (!all_peers_reachable(ngpu, devices))
        return fail(B2G_ERR_UNSUPPORTED,
                    "the fused all-gather needs direct peer access between every pair of devices");
    return for_each_device(ngpu, devices, [&](int g) -> int {
        if (int rc = enable_peers_from(devices[g], ngpu, devices)) return rc;
        int r0, r1;
        panel_rows(M, ngpu, g, r0, r1);
        const size_t off = (size_t)r0 * (size_t)ldd * 2;  // this panel's first row, in bytes
        PeerDst peers;
        for (int h = 0; h < ngpu; ++h)
            if (h != g) peers.ptr[peers.n++] = static_cast<char*>(D_full[h]) + off;
        void* s = streams ? streams[g] : nullptr;
        int rc = gemm_to_peers(A[g], B[g], static_cast<char*>(D_full[g]) + off,
                               bias ? bias[g] : nullptr, r1 - r0, N, K, lda, ldb, ldd, b_layout,
                               acc, epilogue, alpha, tile, stages, group, s, peers);
        if (rc == B2G_OK && sync) rc = b2g_sync_status(s);
        return rc;
    });
}

B2G_EXPORT int b2g_gemm_peers(const void* A, const void* B, void* D, const void* bias, int M,
                              int N, int K, long long lda, long long ldb, long long ldd,
                              int b_layout, int acc, int epilogue, float alpha, int tile,
                              int stages, int group, const void* const* peer_D, int npeer,
                              void* stream) {
    using namespace b2g;
    clear_error();
    if (npeer < 0 || npeer > kMaxPeerDst)
        return fail(B2G_ERR_ARG, "npeer must be 0..%d, got %d", kMaxPeerDst, npeer);
    if (npeer > 0 && !peer_D) return fail(B2G_ERR_ARG, "peer_D is NULL with npeer = %d", npeer);
    PeerDst peers;
    peers.n = npeer;
    for (int i = 0; i < npeer; ++i) peers.ptr[i] = const_cast<void*>(peer_D[i]);
    return gemm_to_peers(A, B, D, bias, M, N, K, lda, ldb, ldd, b_layout, acc, epilogue, alpha,
                         tile, stages, group, stream, peers);
}

// ---------------------------------------------------------------------------------------
// CUDA IPC: one process per GPU shares its D buffer with the others (fused all-gather).
// ---------------------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");

B2G_EXPORT int b2g_ipc_handle(const void* ptr, void* handle, unsigned long long* offset) {
    using namespace b2g;
    clear_error();
    if (!ptr || !handle || !offset) return fail(B2G_ERR_ARG, "ptr, handle and offset are required");
    static PFN_cuMemGetAddressRange_v3020 range = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    });
    if (!range) return fail(B2G_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = range(&base, &size, (CUdeviceptr)(uintptr_t)ptr);
    if (r != CUDA_SUCCESS)
        return fail(B2G_ERR_ARG, "pointer %p is not device memory (cuMemGetAddressRange: %d)",
                    ptr, (int)r);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, (void*)(uintptr_t)base);
    if (e != cudaSuccess)
        return fail(B2G_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    memcpy(handle, &h, sizeof h);
    *offset = (unsigned long long)((uintptr_t)ptr - (uintptr_t)base);
    return B2G_OK;
}

B2G_EXPORT int b2g_ipc_open(const void* handle, void** base) {
    using namespace b2g;
    clear_error();
    if (!handle || !base) return fail(B2G_ERR_ARG, "handle and base are required");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        *base = nullptr;
        return fail(B2G_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    }
    return B2G_OK;
}

B2G_EXPORT int b2g_ipc_close(void* base) {
    using namespace b2g;
    clear_error();
    if (!base) return fail(B2G_ERR_ARG, "base is NULL");
    cudaError_t e = cudaIpcCloseMemHandle(base);
    return e == cudaSuccess ? B2G_OK
                            : fail(B2G_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
}
