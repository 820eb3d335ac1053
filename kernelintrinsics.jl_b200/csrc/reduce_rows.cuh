// reduce_rows.cuh -- segmented reduce: one result per row of a row-major matrix with a leading
// dimension (Base.sum / prod / maximum / minimum / reduce(|, &, xor) along the contiguous dimension,
// e.g. sum(A; dims=1) of a column-major Julia matrix, one result per column).  The kernels and their
// launch are templates; reduce_rows*.cu instantiate them an operator family per file.
//
// The same operators, types and result types as ki_reduce (ki/ops.cuh).  Two kernels:
//   * short rows (cols <= 2048): persistent warps, folding rows of up to 1 KiB 4 at a time and longer
//     ones one at a time (16-byte vectors when the rows allow, lanes striding the row) with
//     __shfl_xor_sync (@warpfold);
//   * long rows: each row is cut into chunks, one 256-thread block per chunk streams it (16-byte
//     vectors when the rows allow, 4 in flight per thread), folds it like the device-wide reduce and
//     writes a partial; the last block of a row (per-row atomic ticket after a release fence) folds
//     the row's partials in order.  Chunks per row are chosen so the grid fills the GPU even when
//     there are few rows.
// Both are deterministic for a given shape and device.
// Folding 1-byte vectors lane-wise (SWAR, as the device-wide reduce does) gave mixed results here
// (UInt8 | over 2^21 x 256: 0.40 -> 0.51 of the copy peak, Int8 maximum over 16384 x 65536: 0.81 ->
// 0.78), so rows keep the element-by-element fold.
#pragma once

#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/ops.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;
constexpr size_t kShortRow = 2048;  // rows up to this many elements take one warp each

// Short rows: persistent warps.  Rows of at most 1 KiB are taken RPP = 4 at a time so that several
// rows' loads are in flight (a 128-element Float32 row is one 16-byte load per lane); longer rows
// one at a time with 4 vectors per lane in flight.
template <class T, class Op, bool VEC, int RPP>
__global__ void __launch_bounds__(kThreads) rows_warp_kernel(const T* __restrict__ x, size_t rows, size_t cols,
                                                             size_t ld, typename ki::Traits<T, Op>::R* out) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using V = ki::Packed16<T>;
    constexpr int kVec = (int)(16 / sizeof(T));
    const ki::OpFn<T, Op> f;
    const unsigned lane = threadIdx.x & 31;
    const size_t nwarps = (size_t)gridDim.x * kWarps;
    const size_t nvec = VEC ? cols / kVec : 0;
    constexpr int kIn = RPP == 1 ? 4 : 1;  // vectors per lane and row in flight
    for (size_t r0 = ((size_t)blockIdx.x * kWarps + (threadIdx.x >> 5)) * RPP; r0 < rows; r0 += nwarps * RPP) {
        A acc[RPP];
#pragma unroll
        for (int u = 0; u < RPP; ++u) acc[u] = Tr::identity();
        if constexpr (VEC) {  // rows start on 16-byte boundaries
            for (size_t i0 = lane; i0 < nvec; i0 += 32 * kIn) {
                V v[RPP][kIn];
#pragma unroll
                for (int u = 0; u < RPP; ++u)
#pragma unroll
                    for (int q = 0; q < kIn; ++q) {
                        const size_t i = i0 + 32 * q;
                        if (r0 + u < rows && i < nvec) {
                            v[u][q].raw = __ldcs(reinterpret_cast<const uint4*>(x + (r0 + u) * ld) + i);
                        }
                    }
#pragma unroll
                for (int u = 0; u < RPP; ++u)
#pragma unroll
                    for (int q = 0; q < kIn; ++q)
                        if (r0 + u < rows && i0 + 32 * q < nvec)
#pragma unroll
                            for (int e = 0; e < kVec; ++e) acc[u] = Tr::op(acc[u], Tr::lift(v[u][q].get(e)));
            }
        }
        for (size_t c = nvec * kVec + lane; c < cols; c += 32) {
#pragma unroll
            for (int u = 0; u < RPP; ++u)
                if (r0 + u < rows) acc[u] = Tr::op(acc[u], Tr::lift(__ldcs(x + (r0 + u) * ld + c)));
        }
#pragma unroll
        for (int u = 0; u < RPP; ++u) {
            const A a = ki::warpfold(acc[u], f);
            if (lane == 0 && r0 + u < rows) out[r0 + u] = Tr::lower(a);
        }
    }
}

template <class T, class Op, bool VEC>
__global__ void __launch_bounds__(kThreads)
    rows_chunk_kernel(const T* __restrict__ x, size_t cols, size_t ld, size_t chunk, unsigned bpr,
                      typename ki::Traits<T, Op>::A* partials, unsigned int* tickets, typename ki::Traits<T, Op>::R* out) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using V = ki::Packed16<T>;
    constexpr int kVec = (int)(16 / sizeof(T));
    const ki::OpFn<T, Op> f;
    const A id = Tr::identity();
    __shared__ A sm[kWarps];
    __shared__ int is_last;
    const size_t row = blockIdx.x / bpr;
    const unsigned part = blockIdx.x % bpr;
    const size_t c0 = (size_t)part * chunk;
    const size_t c1 = c0 + chunk < cols ? c0 + chunk : cols;
    const T* xr = x + row * ld;
    A acc = id;
    if constexpr (VEC) {  // row start, ld and chunk are multiples of 16 bytes
        const uint4* xv = reinterpret_cast<const uint4*>(xr + c0);
        const size_t nv = (c1 - c0) / kVec;
        size_t i = threadIdx.x;
        for (; i + (kUnroll - 1) * kThreads < nv; i += kUnroll * kThreads) {
            V v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                v[u].raw = __ldcs(xv + i + u * kThreads);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
#pragma unroll
                for (int e = 0; e < kVec; ++e) acc = Tr::op(acc, Tr::lift(v[u].get(e)));
        }
        for (; i < nv; i += kThreads) {
            V v;
            v.raw = __ldcs(xv + i);
#pragma unroll
            for (int e = 0; e < kVec; ++e) acc = Tr::op(acc, Tr::lift(v.get(e)));
        }
        for (size_t c = c0 + nv * kVec + threadIdx.x; c < c1; c += kThreads) acc = Tr::op(acc, Tr::lift(xr[c]));
    } else {
        for (size_t c = c0 + threadIdx.x; c < c1; c += kThreads) acc = Tr::op(acc, Tr::lift(__ldcs(xr + c)));
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    acc = ki::warpfold(acc, f);
    if (lane == 0) sm[w] = acc;
    __syncthreads();
    if (w == 0) {
        A b = (lane < kWarps) ? sm[lane] : id;
        b = ki::warpfold(b, f);
        if (lane == 0) {
            partials[row * bpr + part] = b;
            ki::fence<ki::Scope::Device, ki::Order::AcqRel>();
            is_last = atomicAdd(&tickets[row], 1u) == bpr - 1;
        }
    }
    __syncthreads();
    if (!is_last) return;
    ki::fence<ki::Scope::Device, ki::Order::AcqRel>();
    if (w == 0) {
        A r = id;
        for (unsigned b = lane; b < bpr; b += 32)
            r = Tr::op(r, ki::load<ki::Order::Relaxed, ki::Scope::Device>(partials + row * bpr + b));
        r = ki::warpfold(r, f);
        if (lane == 0) {
            out[row] = Tr::lower(r);
            tickets[row] = 0u;  // ready for the next call on this stream
        }
    }
}

template <class T, class Op>
int rows_launch(ki_ctx* ctx, const void* d_x, size_t rows, size_t cols, size_t ld, void* d_out, cudaStream_t s) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    constexpr int kVec = (int)(16 / sizeof(T));
    if (!ki::aligned(d_x, sizeof(T)) || !ki::aligned(d_out, sizeof(R)))
        return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: misaligned input or output");
    const T* x = static_cast<const T*>(d_x);
    R* out = static_cast<R*>(d_out);
    if (cols <= kShortRow) {
        const bool vec = ki::aligned(d_x, 16) && (ld * sizeof(T)) % 16 == 0;
        const bool multi = cols * sizeof(T) <= 1024;
        const size_t rpp = multi ? 4 : 1;
        size_t blocks = (rows + (size_t)kWarps * rpp - 1) / ((size_t)kWarps * rpp);
        const size_t max_blocks = (size_t)ctx->sm_count * 8;
        if (blocks > max_blocks) blocks = max_blocks;
        const unsigned g = (unsigned)blocks;
        if (vec && multi) rows_warp_kernel<T, Op, true, 4><<<g, kThreads, 0, s>>>(x, rows, cols, ld, out);
        else if (vec) rows_warp_kernel<T, Op, true, 1><<<g, kThreads, 0, s>>>(x, rows, cols, ld, out);
        else if (multi) rows_warp_kernel<T, Op, false, 4><<<g, kThreads, 0, s>>>(x, rows, cols, ld, out);
        else rows_warp_kernel<T, Op, false, 1><<<g, kThreads, 0, s>>>(x, rows, cols, ld, out);
        return ki::check_launch(ctx, "rows_warp_kernel launch");
    }
    // chunks per row: fill ~8 blocks per SM, but keep each chunk at least 4 vectors per thread
    const size_t min_chunk = (size_t)kThreads * kUnroll * kVec;
    size_t bpr = ((size_t)ctx->sm_count * 8 + rows - 1) / rows;
    const size_t max_bpr = (cols + min_chunk - 1) / min_chunk;
    if (bpr > max_bpr) bpr = max_bpr;
    if (bpr < 1) bpr = 1;
    size_t chunk = (cols + bpr - 1) / bpr;
    chunk = (chunk + kVec - 1) / kVec * kVec;  // whole vectors
    bpr = (cols + chunk - 1) / chunk;
    // Per-row tickets live in a region of their own: it only ever holds tickets, which start at zero
    // (a new region is cleared) and are reset by each row's last block, so no clearing per call.
    void* tbase = nullptr;
    void* pbase = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_ROWS, rows * sizeof(unsigned), &tbase);
    if (rc) return rc;
    rc = ki::ensure_region(ctx, KI_REG_ROWS_PART, rows * bpr * sizeof(A), &pbase);
    if (rc) return rc;
    unsigned* tickets = static_cast<unsigned*>(tbase);
    A* partials = static_cast<A*>(pbase);
    const bool vec = ki::aligned(d_x, 16) && (ld * sizeof(T)) % 16 == 0;
    if (rows * bpr > 0x7fffffffull) return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: matrix too large");
    const unsigned grid = (unsigned)(rows * bpr);
    if (vec) rows_chunk_kernel<T, Op, true><<<grid, kThreads, 0, s>>>(x, cols, ld, chunk, (unsigned)bpr, partials, tickets, out);
    else rows_chunk_kernel<T, Op, false><<<grid, kThreads, 0, s>>>(x, cols, ld, chunk, (unsigned)bpr, partials, tickets, out);
    return ki::check_launch(ctx, "rows_chunk_kernel launch");
}

template <class Op>
int rows_op(ki_ctx* ctx, int dtype, const void* d_x, size_t rows, size_t cols, size_t ld, void* d_out, cudaStream_t s) {
    constexpr int kBad = -1000;
    const int rc = ki::with_dtype(dtype, kBad, [&](auto tag) -> int {
        using T = decltype(tag);
        if constexpr (ki::op_takes<T, Op>()) return rows_launch<T, Op>(ctx, d_x, rows, cols, ld, d_out, s);
        else return kBad;
    });
    if (rc == kBad) return ki::set_error(ctx, KI_ERR_ARG, "reduce_rows: the operator does not take this element type");
    return rc;
}

}  // namespace

// One per operator, defined in reduce_rows*.cu.
#define KI_ROWS_ENTRY(name)                                                                                      \
    __attribute__((visibility("hidden"))) int name(ki_ctx* ctx, int dtype, const void* d_x, size_t rows, size_t cols, \
                                                   size_t ld, void* d_out, cudaStream_t s)
KI_ROWS_ENTRY(ki_rows_add);
KI_ROWS_ENTRY(ki_rows_mul);
KI_ROWS_ENTRY(ki_rows_max);
KI_ROWS_ENTRY(ki_rows_min);
KI_ROWS_ENTRY(ki_rows_or);
KI_ROWS_ENTRY(ki_rows_and);
KI_ROWS_ENTRY(ki_rows_xor);
