// b2g_internal.h -- state shared by the device translation unit (b2g_kernels.cu) and the
// host-only one (b2g_host.cpp): error reporting, the wait limit, per-device facts.
#pragma once

#include <cstdarg>
#include <cstdint>

#define B2G_EXPORT extern "C" __attribute__((visibility("default")))

namespace b2g {

// Records a formatted message as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

// Device-side wait limit in nanoseconds (b2g_set_wait_timeout_us / B2G_WAIT_TIMEOUT_US).
unsigned long long wait_timeout_ns();

struct DeviceInfo {
    int device = -1;
    int major = 0, minor = 0;
    int sm_count = 0;
    int smem_optin = 0;   // max dynamic shared memory per block (opt-in)
    int smem_per_sm = 0;  // shared memory per SM
};

// Facts about the current device, cached. Returns B2G_OK or an error (with message).
int current_device(DeviceInfo& out);

// Extra copies of a GEMM's D for a fused all-gather: ptr[i] addresses D's first row in a
// copy on another device (peer access enabled), with D's ldd.
constexpr int kMaxPeerDst = 7;
struct PeerDst {
    int n = 0;
    void* ptr[kMaxPeerDst] = {};
};

// b2g_gemm on the current device whose epilogue also writes every D element into each
// peers.ptr[i] (requires N % 8 == 0, ldd % 8 == 0, D and the copies 16-byte aligned).
int gemm_to_peers(const void* A, const void* B, void* D, const void* bias, int M, int N, int K,
                  long long lda, long long ldb, long long ldd, int b_layout, int acc,
                  int epilogue, float alpha, int tile, int stages, int group, void* stream,
                  const PeerDst& peers);

// Copies `rows` x N of a D panel (pitch ldd) into each dst[i] (same pitch) with 16-byte
// loads and stores on the current device (peer destinations over NVLink). Requires N % 8 ==
// 0, ldd % 8 == 0 and 16-byte aligned pointers; 1..8 destinations.
constexpr int kMaxGatherDst = 8;
int allgather_push(const void* src, int rows, int N, long long ldd, void* const* dst, int ndst,
                   void* stream);

}  // namespace b2g
