// ctx.cu -- library version, device queries and the per-device context.
//
// Device queries restate src/device.jl:1-19 and ext/CUDA/device.jl:4-13 (devices, device
// selection, get_warpsize).  The context owns the per-operation scratch and the device status
// word that bounded device-side waits latch into.
#include "ki/common.cuh"

extern "C" {

int ki_version(void) { return 100; }  // 0.1.0

const char* ki_status_string(int status) {
    switch (status) {
        case KI_OK: return "KI_OK";
        case KI_ERR_ARG: return "KI_ERR_ARG: invalid argument";
        case KI_ERR_CUDA: return "KI_ERR_CUDA: CUDA runtime error";
        case KI_ERR_TIMEOUT: return "KI_ERR_TIMEOUT: a bounded device-side wait ran out";
        case KI_ERR_UNSUPPORTED: return "KI_ERR_UNSUPPORTED: device or feature not supported";
        case KI_ERR_NOMEM: return "KI_ERR_NOMEM: scratch allocation failed";
        case KI_ERR_NCCL: return "KI_ERR_NCCL: an NCCL call failed";
        default: return "unknown ki_status";
    }
}

int ki_device_count(int* count) {
    if (!count) return KI_ERR_ARG;
    cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        *count = 0;
        return KI_ERR_CUDA;
    }
    return KI_OK;
}

int ki_device_info(int device, int* sm_count, int* warp_size, int* cc_major, int* cc_minor) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return KI_ERR_CUDA;
    if (sm_count) *sm_count = p.multiProcessorCount;
    if (warp_size) *warp_size = p.warpSize;
    if (cc_major) *cc_major = p.major;
    if (cc_minor) *cc_minor = p.minor;
    return KI_OK;
}

int ki_ctx_create(int device, ki_ctx** out) {
    if (!out) return KI_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return KI_ERR_ARG;
    ki_ctx* ctx = new (std::nothrow) ki_ctx();
    if (!ctx) return KI_ERR_NOMEM;
    ctx->device = device;
    ki::DeviceGuard g(device);
    if (!g.ok) {
        delete ctx;
        return KI_ERR_CUDA;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) {
        delete ctx;
        return KI_ERR_CUDA;
    }
    ctx->sm_count = p.multiProcessorCount;
    ctx->cc_major = p.major;
    ctx->cc_minor = p.minor;
    ctx->max_smem_optin = (int)p.sharedMemPerBlockOptin;
    if (p.major != 10) {
        delete ctx;
        return KI_ERR_UNSUPPORTED;  // the kernels are built for sm_100a only
    }
    if (cudaMalloc(&ctx->d_status, sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(ctx->d_status, 0, sizeof(uint32_t)) != cudaSuccess) {
        if (ctx->d_status) cudaFree(ctx->d_status);
        delete ctx;
        return KI_ERR_NOMEM;
    }
    *out = ctx;
    return KI_OK;
}

int ki_ctx_destroy(ki_ctx* ctx) {
    if (!ctx) return KI_OK;
    {
        ki::DeviceGuard g(ctx->device);
        cudaDeviceSynchronize();
        for (int i = 0; i < KI_PIPE_SLOTS; ++i) {
            if (ctx->pipe_landed[i]) cudaEventDestroy(ctx->pipe_landed[i]);
            if (ctx->pipe_copied[i]) cudaEventDestroy(ctx->pipe_copied[i]);
            if (ctx->pipe_drained[i]) cudaEventDestroy(ctx->pipe_drained[i]);
        }
        if (ctx->pipe_begin) cudaEventDestroy(ctx->pipe_begin);
        if (ctx->pipe_end) cudaEventDestroy(ctx->pipe_end);
        for (int i = 0; i < 3; ++i)
            if (ctx->pipe_stream[i]) cudaStreamDestroy(ctx->pipe_stream[i]);
        for (int r = 0; r < KI_REG_COUNT; ++r)
            if (ctx->region[r]) cudaFree(ctx->region[r]);
        if (ctx->d_status) cudaFree(ctx->d_status);
    }
    delete ctx;
    return KI_OK;
}

const char* ki_last_error_string(const ki_ctx* ctx) {
    if (ctx) return ctx->last_error;
    const char* t = ki::thread_error();
    return t[0] ? t : "null context";
}

int ki_ctx_set_wait_timeout_ns(ki_ctx* ctx, uint64_t ns) {
    KI_CHECK_CTX(ctx);
    if (ns == 0) return ki::set_error(ctx, KI_ERR_ARG, "wait timeout must be positive");
    ctx->wait_timeout_ns = ns;
    return KI_OK;
}

int ki_ctx_check(ki_ctx* ctx, void* stream) {
    KI_CHECK_CTX(ctx);
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    KI_CUDA(ctx, cudaStreamSynchronize(s));
    uint32_t st = 0;
    KI_CUDA(ctx, cudaMemcpy(&st, ctx->d_status, sizeof(st), cudaMemcpyDeviceToHost));
    if (st) {
        KI_CUDA(ctx, cudaMemset(ctx->d_status, 0, sizeof(uint32_t)));
        if (st & KI_DEV_TIMEOUT)
            return ki::set_error(ctx, KI_ERR_TIMEOUT, "a device-side wait ran out (status 0x%x)", st);
        return ki::set_error(ctx, KI_ERR_CUDA, "device reported an inconsistent state (status 0x%x)", st);
    }
    return KI_OK;
}

}  // extern "C"
