// reduce.cuh -- grid-wide reduce (Base.sum / prod / maximum / minimum / reduce(|, &, xor)) built from
// @warpfold-style folds.
//
// One launch: every thread streams 16-byte vectors (several loads in flight), folds them into a
// per-thread accumulator, the warp folds with __shfl_xor_sync (every lane holds the warp total;
// src/warp.jl:273-282 is the reference's Down form, whose lane 1 holds the same total), warps
// combine through a shared-memory tree and each block writes one partial.  The last block to
// finish (atomic ticket after a device-scope release fence) folds the partials in a fixed order and
// writes the result, so the result is deterministic for a given n and device.
//
// Launches use programmatic dependent launch (griddepcontrol): every block waits for the previous
// kernel in the stream to complete before it reads or writes anything, but before that wait it
// issues L2 prefetches of its first vectors, and it releases the next launch at once.  Back to back
// (a CUDA graph of 2^24-element sums over rotating inputs) a launch then takes 11.8 us instead of
// 13.2: the next launch's dispatch and first DRAM reads overlap this one's last-block fold, when the
// DRAM would otherwise be idle (without the prefetches: 13.0 us).  After a kernel that does not
// release its dependents early the launch behaves as an ordinary one.
//
// Operators and types follow Julia Base (ki/ops.cuh): Float32 sums accumulate in Float64 once each
// 16-byte vector has been added in Float32 (within a few ulps of a Float64 sum; the parity bound is
// 1e-5*log2(n) relative), sums and products of integers narrower than 64 bits widen to 64 bits,
// 64-bit ones wrap, maximum/minimum propagate NaN and order signed zeros as Base.max/Base.min do,
// and the bitwise operators take integers in their own type.
#pragma once

#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/ops.cuh"

namespace {

#ifndef KI_REDUCE_PDL
#define KI_REDUCE_PDL 1
#endif
#ifndef KI_REDUCE_PDL_PREFETCH
#define KI_REDUCE_PDL_PREFETCH 1
#endif
#ifndef KI_REDUCE_THREADS
#define KI_REDUCE_THREADS 256
#endif
#ifndef KI_REDUCE_UNROLL
#define KI_REDUCE_UNROLL 4
#endif
#ifndef KI_REDUCE_TAIL_BATCH
#define KI_REDUCE_TAIL_BATCH 1
#endif
#ifndef KI_REDUCE_FOLD_BATCH
#define KI_REDUCE_FOLD_BATCH 8
#endif
#ifndef KI_REDUCE_BLOCKS_PER_SM
#define KI_REDUCE_BLOCKS_PER_SM 8
#endif
constexpr int kThreads = KI_REDUCE_THREADS;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = KI_REDUCE_UNROLL;          // 16-byte loads in flight per thread
constexpr int kBlocksPerSm = KI_REDUCE_BLOCKS_PER_SM;

// Fold of one 16-byte vector into the accumulation type.  Float32 sums add the four lanes in
// Float32 first (one rounding per vector), everything else folds in the accumulation type.
template <class T, class Op, class M>
__device__ __forceinline__ typename ki::Traits<T, Op>::A fold_vec(const ki::Packed16<T>& v) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    constexpr int kV = (int)(16 / sizeof(T));
    if constexpr (std::is_same<T, float>::value && std::is_same<Op, ki::JAdd>::value) {
        return (double)((M::apply(v.get(0)) + M::apply(v.get(1))) + (M::apply(v.get(2)) + M::apply(v.get(3))));
    } else if constexpr (std::is_same<M, ki::MapId>::value && ki::swar_on<T, Op>()) {
        // 1- and 2-byte elements that keep their type: the four words are combined lane-wise
        // (SWAR), then the lanes of the one word left
        using SW = ki::Swar<T, Op>;
        uint32_t w = SW::comb(SW::comb(v.raw.x, v.raw.y), SW::comb(v.raw.z, v.raw.w));
#pragma unroll
        for (int sh = 16; sh >= SW::kBits; sh >>= 1) w = SW::comb(w, (w >> sh) | (SW::kId & ~(0xFFFFFFFFu >> sh)));
        return (A)(T)(w & SW::kMask);
    } else {
        A r = Tr::lift(M::apply(v.get(0)));
#pragma unroll
        for (int i = 1; i < kV; ++i) r = Tr::op(r, Tr::lift(M::apply(v.get(i))));
        return r;
    }
}

template <class A, class F>
__device__ __forceinline__ A block_fold(A v, A* sm, F f, A id) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = ki::warpfold(v, f);
    if (lane == 0) sm[w] = v;
    __syncthreads();
    A r = id;
    if (w == 0) {
        r = (lane < kWarps) ? sm[lane] : id;
        r = ki::warpfold(r, f);
    }
    return r;  // valid in warp 0
}

template <class T, class Op, class M>
__global__ void __launch_bounds__(kThreads)
    reduce_kernel(const T* __restrict__ x, size_t head, size_t nvec, size_t n, typename ki::Traits<T, Op>::A* partials,
                  unsigned int* ticket, typename ki::Traits<T, Op>::R* out, typename ki::Traits<T, Op>::A* out_acc) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using V = ki::Packed16<T>;
    constexpr int kVec = (int)(16 / sizeof(T));
    const ki::OpFn<T, Op> f;
    const A id = Tr::identity();
    __shared__ A sm[kWarps];
    __shared__ int is_last;

    const uint4* xv = reinterpret_cast<const uint4*>(x + head);
    const size_t stride = (size_t)gridDim.x * kThreads;
    size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
#if KI_REDUCE_PDL
    // launched with programmatic stream serialization: the launch and block dispatch overlap the
    // previous kernel's tail.  Nothing is read or written before that kernel has completed; only L2
    // prefetches of this thread's first vectors (hints without effect on the values read) go first.
#if KI_REDUCE_PDL_PREFETCH
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
        if (i + u * stride < nvec) asm volatile("prefetch.global.L2 [%0];" ::"l"(xv + i + u * stride));
#endif
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
    A acc = id;
    for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
        V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            v[u].raw = __ldcs(xv + i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) acc = Tr::op(acc, fold_vec<T, Op, M>(v[u]));
    }
#if KI_REDUCE_TAIL_BATCH
    {  // the last (fewer than kUnroll) vectors of this thread, requested together
        V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            if (i + u * stride < nvec) v[u].raw = __ldcs(xv + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            if (i + u * stride < nvec) acc = Tr::op(acc, fold_vec<T, Op, M>(v[u]));
    }
#else
    for (; i < nvec; i += stride) {
        V v;
        v.raw = __ldcs(xv + i);
        acc = Tr::op(acc, fold_vec<T, Op, M>(v));
    }
#endif
    // unaligned head and the tail that does not fill a vector
    if (blockIdx.x == 0) {
        const size_t tail0 = head + nvec * kVec;
        const int t = threadIdx.x;
        if ((size_t)t < head) acc = Tr::op(acc, Tr::lift(M::apply(x[t])));
        if ((size_t)t < n - tail0) acc = Tr::op(acc, Tr::lift(M::apply(x[tail0 + t])));
    }
    A bsum = block_fold(acc, sm, f, id);
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = bsum;
        ki::fence<ki::Scope::Device, ki::Order::AcqRel>();
        const unsigned prev = atomicAdd(ticket, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    ki::fence<ki::Scope::Device, ki::Order::AcqRel>();
    A r = id;
#if KI_REDUCE_FOLD_BATCH > 1
    // all of a thread's partials requested before any is folded (one L2 round trip, not one per
    // partial); the fold order is the same as one at a time: b = tid, tid + kThreads, ...
    for (unsigned b0 = 0; b0 < gridDim.x; b0 += KI_REDUCE_FOLD_BATCH * kThreads) {
        A v[KI_REDUCE_FOLD_BATCH];
#pragma unroll
        for (int u = 0; u < KI_REDUCE_FOLD_BATCH; ++u) {
            const unsigned b = b0 + (unsigned)u * kThreads + threadIdx.x;
            v[u] = b < gridDim.x ? ki::load<ki::Order::Relaxed, ki::Scope::Device>(partials + b) : id;
        }
#pragma unroll
        for (int u = 0; u < KI_REDUCE_FOLD_BATCH; ++u) r = Tr::op(r, v[u]);
    }
#else
    for (unsigned b = threadIdx.x; b < gridDim.x; b += kThreads)
        r = Tr::op(r, ki::load<ki::Order::Relaxed, ki::Scope::Device>(partials + b));
#endif
    __syncthreads();  // sm reuse
    r = block_fold(r, sm, f, id);
    if (threadIdx.x == 0) {
        if (out_acc) *out_acc = r;
        if (out) *out = Tr::lower(r);
        *ticket = 0u;  // ready for the next call on this stream
    }
}

template <class T, class Op, class M = ki::MapId>
int launch_reduce(ki_ctx* ctx, const T* x, size_t n, typename ki::Traits<T, Op>::R* out,
                  typename ki::Traits<T, Op>::A* out_acc, cudaStream_t s) {
    using A = typename ki::Traits<T, Op>::A;
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
#if KI_REDUCE_PDL
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KI_CUDA(ctx, cudaLaunchKernelEx(&cfg, reduce_kernel<T, Op, M>, static_cast<const T*>(x), head, nvec, n, partials,
                                    ticket, out, out_acc));
    return KI_OK;
#else
    reduce_kernel<T, Op, M><<<(unsigned)blocks, kThreads, 0, s>>>(x, head, nvec, n, partials, ticket, out, out_acc);
    return ki::check_launch(ctx, "reduce_kernel launch");
#endif
}

template <class T, class Op, class M = ki::MapId>
int reduce_generic(ki_ctx* ctx, const void* d_x, size_t n, void* d_out, cudaStream_t s) {
    using R = typename ki::Traits<T, Op>::R;
    if (n > 0 && !ki::aligned(d_x, sizeof(T))) return ki::set_error(ctx, KI_ERR_ARG, "reduce: misaligned input");
    if (!ki::aligned(d_out, sizeof(R))) return ki::set_error(ctx, KI_ERR_ARG, "reduce: misaligned output");
    // n = 0: + and * give their identity (the kernel reads nothing); the others have none (Base throws)
    if (n == 0 && !std::is_same<Op, ki::JAdd>::value && !std::is_same<Op, ki::JMul>::value)
        return ki::set_error(ctx, KI_ERR_ARG, "reduce: reducing an empty collection with an operator that has no identity");
    return launch_reduce<T, Op, M>(ctx, static_cast<const T*>(d_x), n, static_cast<R*>(d_out), nullptr, s);
}

template <class Op, class M = ki::MapId>
int reduce_dtype(ki_ctx* ctx, int dtype, const void* d_x, size_t n, void* d_out, cudaStream_t s) {
    constexpr int kBad = -1000;
    const int rc = ki::with_dtype(dtype, kBad, [&](auto tag) -> int {
        using T = decltype(tag);
        if constexpr (ki::op_takes<T, Op>()) return reduce_generic<T, Op, M>(ctx, d_x, n, d_out, s);
        else return kBad;
    });
    if (rc == kBad) return ki::set_error(ctx, KI_ERR_ARG, "reduce: the operator does not take this element type");
    return rc;
}

}  // namespace

// mapreduce(abs, op, x) and mapreduce(abs2, op, x) for op in +, max, min (reduce_map.cu).
__attribute__((visibility("hidden"))) int ki_reduce_mapped(ki_ctx* ctx, int map, int op, int dtype, const void* d_x,
                                                           size_t n, void* d_out, cudaStream_t s);
