// reduce.cu -- grid-wide sum (Base.sum) built from @warpfold-style folds.
//
// One launch: every thread streams 16-byte vectors (several loads in flight), folds them into a
// per-thread accumulator, the warp folds with __shfl_xor_sync (every lane holds the warp total;
// src/warp.jl:273-282 is the reference's Down form, whose lane 1 holds the same total), warps
// combine through a shared-memory tree and each block writes one partial.  The last block to
// finish (atomic ticket after a device-scope release fence) folds the partials in a fixed order and
// writes the result, so the result is deterministic for a given n and device.
//
// Float32 input accumulates in Float64 once each 16-byte vector has been added in Float32, so the
// result is within a few ulps of a Float64 sum (the parity bound is 1e-5*log2(n) relative).
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"

namespace {

#ifndef KI_REDUCE_THREADS
#define KI_REDUCE_THREADS 256
#endif
#ifndef KI_REDUCE_UNROLL
#define KI_REDUCE_UNROLL 4
#endif
#ifndef KI_REDUCE_BLOCKS_PER_SM
#define KI_REDUCE_BLOCKS_PER_SM 8
#endif
constexpr int kThreads = KI_REDUCE_THREADS;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = KI_REDUCE_UNROLL;          // 16-byte loads in flight per thread
constexpr int kBlocksPerSm = KI_REDUCE_BLOCKS_PER_SM;

template <class T>
struct Acc;
template <>
struct Acc<float> {
    using type = double;
    __device__ static __forceinline__ double vec(const float4& v) { return (double)((v.x + v.y) + (v.z + v.w)); }
    __device__ static __forceinline__ double one(float v) { return (double)v; }
    __device__ static __forceinline__ double add(double a, double b) { return a + b; }
};
template <>
struct Acc<int64_t> {
    using type = int64_t;
    __device__ static __forceinline__ int64_t vec(const longlong2& v) { return ki::wrap_add(v.x, v.y); }
    __device__ static __forceinline__ int64_t one(int64_t v) { return v; }
    __device__ static __forceinline__ int64_t add(int64_t a, int64_t b) { return ki::wrap_add(a, b); }
};

template <class T>
struct Vec;
template <>
struct Vec<float> {
    using type = float4;
};
template <>
struct Vec<int64_t> {
    using type = longlong2;
};

struct AddOp {
    template <class A>
    __device__ __forceinline__ A operator()(A a, A b) const {
        if constexpr (std::is_same<A, int64_t>::value) return ki::wrap_add(a, b);
        else return a + b;
    }
};

template <class A>
__device__ __forceinline__ A block_fold(A v, A* sm) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = ki::warpfold(v, AddOp{});
    if (lane == 0) sm[w] = v;
    __syncthreads();
    A r = A(0);
    if (w == 0) {
        r = (lane < kWarps) ? sm[lane] : A(0);
        r = ki::warpfold(r, AddOp{});
    }
    return r;  // valid in warp 0
}

template <class T>
__global__ void __launch_bounds__(kThreads) reduce_kernel(const T* __restrict__ x, size_t head, size_t nvec,
                                                          size_t n, typename Acc<T>::type* partials,
                                                          unsigned int* ticket, float* out_f32,
                                                          typename Acc<T>::type* out_acc) {
    using A = typename Acc<T>::type;
    using V = typename Vec<T>::type;
    constexpr int kVec = (int)(16 / sizeof(T));
    __shared__ A sm[kWarps];
    __shared__ int is_last;

    const V* xv = reinterpret_cast<const V*>(x + head);
    const size_t stride = (size_t)gridDim.x * kThreads;
    size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    A acc = A(0);
    for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
        V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = __ldcs(xv + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) acc = Acc<T>::add(acc, Acc<T>::vec(v[u]));
    }
    for (; i < nvec; i += stride) acc = Acc<T>::add(acc, Acc<T>::vec(__ldcs(xv + i)));
    // unaligned head and the tail that does not fill a vector
    if (blockIdx.x == 0) {
        const size_t tail0 = head + nvec * kVec;
        const int t = threadIdx.x;
        if ((size_t)t < head) acc = Acc<T>::add(acc, Acc<T>::one(x[t]));
        if ((size_t)t < n - tail0) acc = Acc<T>::add(acc, Acc<T>::one(x[tail0 + t]));
    }
    A bsum = block_fold(acc, sm);
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = bsum;
        ki::fence<ki::Scope::Device, ki::Order::AcqRel>();
        const unsigned prev = atomicAdd(ticket, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    ki::fence<ki::Scope::Device, ki::Order::AcqRel>();
    A r = A(0);
    for (unsigned b = threadIdx.x; b < gridDim.x; b += kThreads)
        r = Acc<T>::add(r, ki::load<ki::Order::Relaxed, ki::Scope::Device>(partials + b));
    __syncthreads();  // sm reuse
    r = block_fold(r, sm);
    if (threadIdx.x == 0) {
        if (out_acc) *out_acc = r;
        if (out_f32) *out_f32 = (float)r;
        *ticket = 0u;  // ready for the next call on this stream
    }
}

template <class T>
int launch_reduce(ki_ctx* ctx, const T* x, size_t n, float* out_f32, typename Acc<T>::type* out_acc,
                  cudaStream_t s) {
    using A = typename Acc<T>::type;
    constexpr int kVec = (int)(16 / sizeof(T));
    size_t head = (size_t)((16 - (reinterpret_cast<uintptr_t>(x) & 15)) & 15) / sizeof(T);
    if (head > n) head = n;
    const size_t nvec = (n - head) / kVec;
    size_t blocks = (nvec + (size_t)kThreads * kUnroll - 1) / ((size_t)kThreads * kUnroll);
    const size_t max_blocks = (size_t)ctx->sm_count * kBlocksPerSm;
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    // scratch: [ticket (256 B)] [partials]
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_REDUCE, 256 + max_blocks * sizeof(A), &base);
    if (rc) return rc;
    unsigned int* ticket = reinterpret_cast<unsigned int*>(base);
    A* partials = reinterpret_cast<A*>(static_cast<char*>(base) + 256);
    reduce_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(x, head, nvec, n, partials, ticket, out_f32, out_acc);
    return ki::check_launch(ctx, "reduce_kernel launch");
}

}  // namespace

extern "C" int ki_reduce_sum_f32(ki_ctx* ctx, const float* d_x, size_t n, float* d_out_f32, double* d_out_f64,
                                 void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_out_f32 && !d_out_f64) return ki::set_error(ctx, KI_ERR_ARG, "reduce: no output");
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "reduce: null input");
    if (n > 0 && !ki::aligned(d_x, 4)) return ki::set_error(ctx, KI_ERR_ARG, "reduce: misaligned Float32 input");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        if (d_out_f32) KI_CUDA(ctx, cudaMemsetAsync(d_out_f32, 0, sizeof(float), s));
        if (d_out_f64) KI_CUDA(ctx, cudaMemsetAsync(d_out_f64, 0, sizeof(double), s));
        return KI_OK;
    }
    return launch_reduce<float>(ctx, d_x, n, d_out_f32, d_out_f64, s);
}

extern "C" int ki_reduce_sum_i64(ki_ctx* ctx, const int64_t* d_x, size_t n, int64_t* d_out, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_out) return ki::set_error(ctx, KI_ERR_ARG, "reduce: no output");
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "reduce: null input");
    if (n > 0 && !ki::aligned(d_x, 8)) return ki::set_error(ctx, KI_ERR_ARG, "reduce: misaligned Int64 input");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        KI_CUDA(ctx, cudaMemsetAsync(d_out, 0, sizeof(int64_t), s));
        return KI_OK;
    }
    return launch_reduce<int64_t>(ctx, d_x, n, nullptr, d_out, s);
}
