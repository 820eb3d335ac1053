// ki/common.cuh -- context, scratch and error plumbing shared by the libki_b200 translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../../include/ki_b200.h"
#include "../../../include/ki/status.h"  // device status bits (read and cleared by ki_ctx_check)

// Scratch regions, one per operation so different operations never share memory.
enum ki_region {
    KI_REG_REDUCE = 0,
    KI_REG_SCAN = 1,
    KI_REG_COMPACT = 2,
    KI_REG_MISC = 3,
    KI_REG_STAGE = 4,  // device staging slots of the host-buffer copy
    KI_REG_SCAN_ANY = 5,  // the generic scan (any operator and type)
    KI_REG_ROWS = 6,       // per-row tickets of the segmented reduce
    KI_REG_ROWS_PART = 7,  // per-row partials of the segmented reduce
    KI_REG_HOST_SHARD = 8, // device copy of a shard for the two-phase sharded host-buffer scan
    KI_REG_HOST_PART = 9,  // per-chunk totals of that scan
    KI_REG_COUNT = 10
};

// Host-buffer pipelines: slots of staging memory cycled over three streams (host -> device,
// kernel, device -> host), KI_PIPE_CHUNK bytes per chunk.
#ifndef KI_PIPE_SLOTS_N
#define KI_PIPE_SLOTS_N 4
#endif
constexpr int KI_PIPE_SLOTS = KI_PIPE_SLOTS_N;
#ifndef KI_PIPE_CHUNK
#define KI_PIPE_CHUNK (16u << 20)
#endif

struct ki_ctx {
    int device = 0;
    int sm_count = 0;
    int max_smem_optin = 0;
    int cc_major = 0, cc_minor = 0;
    uint64_t wait_timeout_ns = 2000000000ull;
    uint32_t* d_status = nullptr;  // device status word (KI_DEV_* bits)
    void* region[KI_REG_COUNT] = {};
    size_t region_bytes[KI_REG_COUNT] = {};
    char last_error[512] = {0};
    int copy_resident[5] = {};  // resident vcopy blocks per SM, per instantiation
    int gemm_pairs = 0;         // co-resident CTA pairs of the pair GEMM kernel
    // host-buffer copy pipeline: streams [0] host -> device, [1] kernel, [2] device -> host
    cudaStream_t pipe_stream[3] = {};
    cudaEvent_t pipe_landed[KI_PIPE_SLOTS] = {};   // slot's input chunk is on the device
    cudaEvent_t pipe_copied[KI_PIPE_SLOTS] = {};   // kernel finished: input read, output written
    cudaEvent_t pipe_drained[KI_PIPE_SLOTS] = {};  // slot's output chunk is back in host memory
    cudaEvent_t pipe_begin = nullptr, pipe_end = nullptr;
};

namespace ki {

// Message of the calling thread's last failed call that had no context to hold it (a communicator
// whose set-up failed); ki_last_error_string(NULL) returns it.
inline char* thread_error() {
    static thread_local char buf[512] = {0};
    return buf;
}

inline int set_error(ki_ctx* ctx, int status, const char* fmt, ...) {
    if (ctx) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(ctx->last_error, sizeof(ctx->last_error), fmt, ap);
        va_end(ap);
    }
    return status;
}

inline int cuda_error(ki_ctx* ctx, cudaError_t e, const char* what) {
    return set_error(ctx, KI_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Make ctx->device current for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = (cudaSetDevice(dev) == cudaSuccess);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Grow a scratch region to at least `bytes` (synchronous cudaMalloc the first time a size is seen).
inline int ensure_region(ki_ctx* ctx, ki_region r, size_t bytes, void** out) {
    if (bytes == 0) bytes = 256;
    if (ctx->region_bytes[r] < bytes) {
        size_t want = bytes + bytes / 8 + 4096;
        if (ctx->region[r]) {
            cudaError_t e = cudaDeviceSynchronize();
            if (e != cudaSuccess) return cuda_error(ctx, e, "cudaDeviceSynchronize (scratch growth)");
            cudaFree(ctx->region[r]);
            ctx->region[r] = nullptr;
            ctx->region_bytes[r] = 0;
        }
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, want);
        if (e != cudaSuccess) return set_error(ctx, KI_ERR_NOMEM, "scratch cudaMalloc(%zu): %s", want,
                                               cudaGetErrorString(e));
        e = cudaMemset(p, 0, want);
        if (e != cudaSuccess) return cuda_error(ctx, e, "cudaMemset (scratch)");
        ctx->region[r] = p;
        ctx->region_bytes[r] = want;
    }
    *out = ctx->region[r];
    return KI_OK;
}

inline int check_launch(ki_ctx* ctx, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(ctx, e, what);
    return KI_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace ki

// Streams and events of the host-buffer pipelines (copy.cu), made on first use.
__attribute__((visibility("hidden"))) int ki_ensure_pipe(ki_ctx* ctx);

#define KI_CHECK_CTX(ctx)                                              \
    do {                                                               \
        if (!(ctx)) return KI_ERR_ARG;                                 \
    } while (0)

#define KI_GUARD(ctx)                                                                     \
    ki::DeviceGuard _ki_guard((ctx)->device);                                             \
    if (!_ki_guard.ok) return ki::set_error((ctx), KI_ERR_CUDA, "cudaSetDevice failed");

#define KI_CUDA(ctx, call)                                   \
    do {                                                     \
        cudaError_t _e = (call);                             \
        if (_e != cudaSuccess) return ki::cuda_error((ctx), _e, #call); \
    } while (0)
