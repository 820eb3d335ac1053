// gen.cu -- seeded synthetic inputs, generated on the device.
//
// Element i of stream `seed` is the (i+1)-th output of splitmix64 started at `seed`:
//     mix64(seed + (i+1) * 0x9E3779B97F4A7C15)
// so any element can be produced independently and the host generator yields the same bits.
#include <cuda_fp8.h>

#include "ki/common.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t rand64(uint64_t seed, uint64_t i) {
    return mix64(seed + (i + 1) * 0x9E3779B97F4A7C15ull);
}
__device__ __forceinline__ float u01(uint64_t r) { return __fmul_rn((float)(r >> 40), 0x1p-24f); }

unsigned grid_for(size_t n) {
    size_t g = (n + kThreads - 1) / kThreads;
    if (g > 148u * 64u) g = 148u * 64u;
    return (unsigned)(g ? g : 1);
}

#define KI_GRID_LOOP(i, n) \
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < (n); i += (size_t)gridDim.x * kThreads)

__global__ void fill_uniform_kernel(uint64_t seed, float* out, size_t n) {
    KI_GRID_LOOP(i, n) out[i] = u01(rand64(seed, i));
}

__global__ void fill_int_kernel(uint64_t seed, int64_t lo, uint64_t span, int64_t* out, size_t n) {
    KI_GRID_LOOP(i, n) out[i] = (int64_t)(rand64(seed, i) % span) + lo;
}

__global__ void fill_bytes_kernel(uint64_t seed, uint8_t* out, size_t n) {
    const size_t words = (n + 7) / 8;
    KI_GRID_LOOP(w, words) {
        const uint64_t r = rand64(seed, w);
        const size_t b0 = w * 8;
        if (b0 + 8 <= n && (((uintptr_t)(out + b0)) & 7) == 0) {
            *reinterpret_cast<uint64_t*>(out + b0) = r;
        } else {
            for (int k = 0; k < 8 && b0 + k < n; ++k) out[b0 + k] = (uint8_t)(r >> (8 * k));
        }
    }
}

// Box-Muller on pairs: z0 = sqrt(-2 ln u1) cos(2 pi u2), z1 = ... sin(...), u1 in (0,1], u2 in [0,1).
__global__ void fill_normal_kernel(uint64_t seed, float* out, size_t n) {
    const size_t pairs = (n + 1) / 2;
    KI_GRID_LOOP(m, pairs) {
        const uint64_t r1 = rand64(seed, 2 * m), r2 = rand64(seed, 2 * m + 1);
        const float a = ((float)(r1 >> 40) + 1.0f) * 0x1p-24f;
        const float b = u01(r2);
        const float rad = sqrtf(-2.0f * logf(a));
        float sn, cs;
        sincospif(2.0f * b, &sn, &cs);
        out[2 * m] = rad * cs;
        if (2 * m + 1 < n) out[2 * m + 1] = rad * sn;
    }
}

// e4m3((2u - 1) * scale), each step rounded to nearest even in binary32, then cvt.rn.satfinite.
__global__ void fill_e4m3_kernel(uint64_t seed, float scale, uint8_t* out, size_t n) {
    KI_GRID_LOOP(i, n) {
        const float u = u01(rand64(seed, i));
        const float c = __fadd_rn(__fmul_rn(2.0f, u), -1.0f);
        const float x = __fmul_rn(c, scale);
        out[i] = (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
    }
}

}  // namespace

extern "C" {

int ki_fill_uniform_f32(ki_ctx* ctx, uint64_t seed, float* d_out, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_out) return KI_ERR_ARG;
    KI_GUARD(ctx);
    fill_uniform_kernel<<<grid_for(n), kThreads, 0, ki::as_stream(stream)>>>(seed, d_out, n);
    return ki::check_launch(ctx, "fill_uniform_kernel");
}

int ki_fill_int_range_i64(ki_ctx* ctx, uint64_t seed, int64_t lo, int64_t hi, int64_t* d_out, size_t n,
                          void* stream) {
    KI_CHECK_CTX(ctx);
    if (hi < lo) return ki::set_error(ctx, KI_ERR_ARG, "fill_int_range: hi < lo");
    if (n == 0) return KI_OK;
    if (!d_out) return KI_ERR_ARG;
    KI_GUARD(ctx);
    const uint64_t span = (uint64_t)hi - (uint64_t)lo + 1;  // 0 means the full 2^64 range
    if (span == 0) return ki::set_error(ctx, KI_ERR_ARG, "fill_int_range: full 64-bit range unsupported");
    fill_int_kernel<<<grid_for(n), kThreads, 0, ki::as_stream(stream)>>>(seed, lo, span, d_out, n);
    return ki::check_launch(ctx, "fill_int_kernel");
}

int ki_fill_bytes(ki_ctx* ctx, uint64_t seed, uint8_t* d_out, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_out) return KI_ERR_ARG;
    KI_GUARD(ctx);
    fill_bytes_kernel<<<grid_for((n + 7) / 8), kThreads, 0, ki::as_stream(stream)>>>(seed, d_out, n);
    return ki::check_launch(ctx, "fill_bytes_kernel");
}

int ki_fill_normal_f32(ki_ctx* ctx, uint64_t seed, float* d_out, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_out) return KI_ERR_ARG;
    KI_GUARD(ctx);
    fill_normal_kernel<<<grid_for((n + 1) / 2), kThreads, 0, ki::as_stream(stream)>>>(seed, d_out, n);
    return ki::check_launch(ctx, "fill_normal_kernel");
}

int ki_fill_e4m3_uniform(ki_ctx* ctx, uint64_t seed, float scale, uint8_t* d_out, size_t n, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_out) return KI_ERR_ARG;
    KI_GUARD(ctx);
    fill_e4m3_kernel<<<grid_for(n), kThreads, 0, ki::as_stream(stream)>>>(seed, scale, d_out, n);
    return ki::check_launch(ctx, "fill_e4m3_kernel");
}

}  // extern "C"
