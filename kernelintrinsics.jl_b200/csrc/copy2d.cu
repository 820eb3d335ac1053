// copy2d.cu -- copyto! between strided views.
//
// The reference moves a strided view (a SubArray that is not dense, a column-major matrix block)
// element by element through the AbstractArray fallbacks of vload / vstore! (_vload_batch /
// _vstore_batch!, src/vectorization.jl:202-211, 290-297, 426-448).  Two device-wide forms here:
//
//   ki_vcopy_2d       height rows of width bytes, row r at src + r*spitch and dst + r*dpitch, any
//                     byte alignment and any pitch (a block of a column-major array: rows = its
//                     columns).  A warp takes one (row, span of 128 16-byte chunks) at a time and
//                     moves it as ki_vcopy moves a whole range: unaligned head and tail bytes, then
//                     aligned 16-byte stores whose source words are re-aligned in registers
//                     (ki/bytes.cuh), so a row misaligned against its destination still reads
//                     whole aligned 16-byte words.  Each row has its own alignment when a pitch is
//                     not a multiple of 16; the word shift is picked per row.  Rows of at most 384
//                     bytes take one thread per 16-byte chunk instead (a warp then spans several
//                     rows).
//   ki_vcopy_strided  count elements with element strides of either sign (view(x, 1:2:n), a row
//                     of a column-major matrix, reverse(view)).  Elements of 1, 2, 4, 8 or 16
//                     bytes: one natural load and store per element, four in flight per thread.
//                     Any other size (a struct of 3, 12 or 40 bytes, which the reference moves
//                     field by field through its scalar fallback): each element as words of the
//                     largest power of two that divides its size (at most 16 bytes), consecutive
//                     threads on consecutive words of an element.
#include "ki/bytes.cuh"
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kSpan = 32 * kUnroll;  // 16-byte chunks per warp item

struct Copy2DArgs {
    uint8_t* dst;
    const uint8_t* src;
    size_t dpitch, spitch, width, height;
    size_t spans;  // warp items per row
};

// One warp item: chunks [sp*kSpan, (sp+1)*kSpan) of a row body of nc chunks at d, whose source
// words start at the aligned address sa (WS, sh: the source's misalignment, as in copy.cu).
template <int WS, bool ALIGNED>
__device__ __forceinline__ void body_span(uint4* __restrict__ d, const uint4* __restrict__ sa, size_t nc, size_t base,
                                          unsigned sh, unsigned lane) {
    if constexpr (ALIGNED) {
        uint4 v[kUnroll];
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const size_t k = base + 32 * j;
            if (k < nc) v[j] = sa[k];
        }
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const size_t k = base + 32 * j;
            if (k < nc) d[k] = v[j];
        }
    } else {
        uint4 lo[kUnroll], ex[kUnroll];
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const size_t k = base + 32 * j;
            lo[j] = make_uint4(0, 0, 0, 0);
            ex[j] = make_uint4(0, 0, 0, 0);
            if (k <= nc) lo[j] = sa[k];  // word nc still holds source bytes of this row
            if (lane == 31 && k < nc) ex[j] = sa[k + 1];
        }
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const size_t k = base + 32 * j;
            uint4 hi = ki::shfl_down_u4(lo[j]);
            if (lane == 31) hi = ex[j];
            if (k < nc) d[k] = ki::realign<WS>(lo[j], hi, sh);
        }
    }
}

__global__ void __launch_bounds__(kThreads) vcopy2d_kernel(Copy2DArgs a) {
    const unsigned lane = threadIdx.x & 31;
    const size_t warp = ((size_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const size_t nwarps = ((size_t)gridDim.x * kThreads) >> 5;
    const size_t items = a.height * a.spans;
    for (size_t it = warp; it < items; it += nwarps) {
        const size_t row = it / a.spans, sp = it - row * a.spans;
        uint8_t* dr = a.dst + row * a.dpitch;
        const uint8_t* sr = a.src + row * a.spitch;
        size_t head = (16 - ((uintptr_t)dr & 15)) & 15;
        if (head > a.width) head = a.width;
        const size_t nc = (a.width - head) / 16;
        if (sp == 0) {  // head and tail bytes (< 16 each)
            const size_t tail = a.width - head - nc * 16, t0 = head + nc * 16;
            if (lane < head) dr[lane] = sr[lane];
            if (lane >= 16 && lane - 16 < tail) dr[t0 + lane - 16] = sr[t0 + lane - 16];
        }
        if (sp * kSpan >= nc) continue;  // the same for the whole warp
        uint4* d = reinterpret_cast<uint4*>(dr + head);
        const uintptr_t sb = (uintptr_t)(sr + head);
        const unsigned mis = (unsigned)(sb & 15);
        const uint4* sa = reinterpret_cast<const uint4*>(sb - mis);
        const unsigned sh = (mis & 3) * 8;
        const size_t base = sp * kSpan + lane;
        switch (mis >> 2) {  // the same for the whole warp (one row)
            case 0:
                if (mis == 0) body_span<0, true>(d, sa, nc, base, sh, lane);
                else body_span<0, false>(d, sa, nc, base, sh, lane);
                break;
            case 1: body_span<1, false>(d, sa, nc, base, sh, lane); break;
            case 2: body_span<2, false>(d, sa, nc, base, sh, lane); break;
            default: body_span<3, false>(d, sa, nc, base, sh, lane); break;
        }
    }
}

// Narrow rows (width <= kNarrowRow bytes): one thread per 16-byte destination chunk instead of one
// warp per row, so a warp covers several rows.  A row owns width/16 + 2 slots: its head bytes, its
// tail bytes and its body chunks.  A body chunk whose source is misaligned reads the two aligned
// source words it straddles (both hold bytes of this row) and re-aligns them in registers; head and
// tail (< 16 bytes each) are copied byte by byte, their loads issued together.  Each thread has
// KI_COPY2D_NARROW_INFLIGHT slots' loads in flight before it stores.  Measured (fraction of the
// copy peak): 64-byte rows 0.34 (one slot at a time 0.24, warp per row 0.08), 100-byte rows 0.28
// (0.24), 256-byte rows 0.36 (0.29, warp per row 0.22), 384-byte rows 0.39 (0.31); 512-byte rows
// run 0.41 warp per row, hence the 384-byte threshold.  Four slots in flight: 0.15-0.29; head and
// tail in a pass of their own after the bodies: faster on aligned rows, slower on short odd ones.
#ifndef KI_COPY2D_NARROW
#define KI_COPY2D_NARROW 384
#endif
constexpr size_t kNarrowRow = KI_COPY2D_NARROW;

template <int WS>
__device__ __forceinline__ uint4 realign_pair(const uint4* sa, unsigned sh) {
    return ki::realign<WS>(sa[0], sa[1], sh);
}

// I: the slot index type (32-bit whenever the slots fit: a 64-bit division per chunk costs more than
// the chunk's copy).
#ifndef KI_COPY2D_NARROW_INFLIGHT
#define KI_COPY2D_NARROW_INFLIGHT 2
#endif

// One row's layout: head bytes before the 16-byte aligned body, nc body chunks.
__device__ __forceinline__ void narrow_row(const Copy2DArgs& a, size_t row, uint8_t*& dr, const uint8_t*& sr,
                                           size_t& head, size_t& nc) {
    dr = a.dst + row * a.dpitch;
    sr = a.src + row * a.spitch;
    head = (16 - ((uintptr_t)dr & 15)) & 15;
    if (head > a.width) head = a.width;
    nc = (a.width - head) / 16;
}

template <class I>
__global__ void __launch_bounds__(kThreads) vcopy2d_narrow_kernel(Copy2DArgs a) {
    constexpr int kIn = KI_COPY2D_NARROW_INFLIGHT;  // slots in flight per thread
    const I n_threads = (I)gridDim.x * kThreads;
    const I slots = (I)(a.width / 16 + 2);  // per row: head bytes, tail bytes, then the body chunks
    const I total = (I)a.height * slots;
    for (I j0 = (I)blockIdx.x * kThreads + threadIdx.x; j0 < total; j0 += n_threads * kIn) {
        uint4 r[kIn];
        uint8_t hv[kIn][15];
        uint8_t* dp[kIn];
        int nb[kIn];  // -1: nothing; 16: a body chunk; 0..15: head or tail bytes
#pragma unroll
        for (int u = 0; u < kIn; ++u) {
            nb[u] = -1;
            const I j = j0 + (I)u * n_threads;
            if (j >= total) continue;
            const I row = j / slots, q = j - row * slots;
            uint8_t* dr;
            const uint8_t* sr;
            size_t head, nc;
            narrow_row(a, (size_t)row, dr, sr, head, nc);
            if (q < 2) {
                const size_t b0 = q == 0 ? 0 : head + nc * 16;
                const int n = (int)(q == 0 ? head : a.width - head - nc * 16);
#pragma unroll
                for (int b = 0; b < 15; ++b)
                    if (b < n) hv[u][b] = sr[b0 + b];
                dp[u] = dr + b0;
                nb[u] = n;
                continue;
            }
            const size_t k = (size_t)q - 2;
            if (k >= nc) continue;
            const uintptr_t sb = (uintptr_t)(sr + head) + 16 * k;
            const unsigned mis = (unsigned)(sb & 15);
            const uint4* sa = reinterpret_cast<const uint4*>(sb - mis);
            const unsigned sh = (mis & 3) * 8;
            switch (mis >> 2) {
                case 0: r[u] = mis == 0 ? sa[0] : realign_pair<0>(sa, sh); break;
                case 1: r[u] = realign_pair<1>(sa, sh); break;
                case 2: r[u] = realign_pair<2>(sa, sh); break;
                default: r[u] = realign_pair<3>(sa, sh); break;
            }
            dp[u] = dr + head + 16 * k;
            nb[u] = 16;
        }
#pragma unroll
        for (int u = 0; u < kIn; ++u) {
            if (nb[u] == 16) {
                *reinterpret_cast<uint4*>(dp[u]) = r[u];
            } else {
#pragma unroll
                for (int b = 0; b < 15; ++b)
                    if (b < nb[u]) dp[u][b] = hv[u][b];
            }
        }
    }
}

template <int B>
struct Word;
template <> struct Word<1> { using type = uint8_t; };
template <> struct Word<2> { using type = uint16_t; };
template <> struct Word<4> { using type = uint32_t; };
template <> struct Word<8> { using type = uint64_t; };
template <> struct Word<16> { using type = uint4; };

template <int B>
__global__ void __launch_bounds__(kThreads) strided_kernel(uint8_t* dst, int64_t dstride, const uint8_t* src,
                                                           int64_t sstride, size_t count) {
    using W = typename Word<B>::type;
    const size_t n_threads = (size_t)gridDim.x * kThreads;
    const size_t t = (size_t)blockIdx.x * kThreads + threadIdx.x;
    for (size_t i0 = t; i0 < count; i0 += n_threads * kUnroll) {
        W v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t i = i0 + (size_t)u * n_threads;
            if (i < count) v[u] = __ldcs(reinterpret_cast<const W*>(src + (int64_t)i * sstride * B));
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t i = i0 + (size_t)u * n_threads;
            if (i < count) __stcs(reinterpret_cast<W*>(dst + (int64_t)i * dstride * B), v[u]);
        }
    }
}

// Elements of nw words of W bytes (element sizes that are not 1, 2, 4, 8 or 16); strides in bytes.
template <int W>
__global__ void __launch_bounds__(kThreads) strided_words_kernel(uint8_t* dst, int64_t dstride_b, const uint8_t* src,
                                                                 int64_t sstride_b, size_t count, unsigned nw) {
    using Wt = typename Word<W>::type;
    const size_t total = count * nw;
    const size_t n_threads = (size_t)gridDim.x * kThreads;
    for (size_t j = (size_t)blockIdx.x * kThreads + threadIdx.x; j < total; j += n_threads) {
        const size_t i = j / nw;
        const size_t q = j - i * nw;
        const Wt v = __ldcs(reinterpret_cast<const Wt*>(src + (int64_t)i * sstride_b + (int64_t)(q * W)));
        __stcs(reinterpret_cast<Wt*>(dst + (int64_t)i * dstride_b + (int64_t)(q * W)), v);
    }
}

size_t grid_for(ki_ctx* ctx, size_t warps_of_work) {
    size_t blocks = (warps_of_work + (kThreads / 32) - 1) / (kThreads / 32);
    const size_t cap = (size_t)ctx->sm_count * (2048 / kThreads);
    if (blocks > cap) blocks = cap;
    return blocks < 1 ? 1 : blocks;
}

// Lowest and one-past-highest byte an (element) range touches.
void span_of(uintptr_t p, int64_t stride_bytes, size_t count, size_t elem, uintptr_t* lo, uintptr_t* hi) {
    const int64_t last = (int64_t)(count - 1) * stride_bytes;
    *lo = last < 0 ? p + last : p;
    *hi = (last < 0 ? p : p + last) + elem;
}

}  // namespace

extern "C" int ki_vcopy_2d(ki_ctx* ctx, void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                           size_t height, void* stream) {
    KI_CHECK_CTX(ctx);
    if (width == 0 || height == 0) return KI_OK;
    if (!dst || !src) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_2d: null pointer");
    if (height > 1 && (dpitch < width || spitch < width))
        return ki::set_error(ctx, KI_ERR_ARG, "vcopy_2d: a pitch is smaller than the row width");
    uintptr_t dl, dh, sl, sh;
    span_of((uintptr_t)dst, (int64_t)dpitch, height, width, &dl, &dh);
    span_of((uintptr_t)src, (int64_t)spitch, height, width, &sl, &sh);
    if (dl < sh && sl < dh) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_2d: source and destination ranges overlap");
    KI_GUARD(ctx);
    Copy2DArgs a;
    a.dst = static_cast<uint8_t*>(dst);
    a.src = static_cast<const uint8_t*>(src);
    a.dpitch = dpitch;
    a.spitch = spitch;
    a.width = width;
    a.height = height;
    a.spans = (width / 16 + kSpan) / kSpan;  // at least one: the item that also moves head and tail
    // narrow rows; and rows up to 1 KiB whose pitches give each row its own alignment (the warp per
    // row then re-aligns every row: 768-byte rows at odd pitches 0.35 of the copy peak that way,
    // 0.46 narrow; equal aligned 1 KiB rows 0.79 warp per row, 0.61 narrow)
    const bool odd_pitch = (dpitch % 16) != 0 || (spitch % 16) != 0;
    if (height > 1 && (width <= kNarrowRow || (width <= 1024 && odd_pitch))) {
        const size_t threads = height * (width / 16 + 2);  // head and tail slots plus the body chunks
        const unsigned g = (unsigned)grid_for(ctx, (threads + 31) / 32);
        // 32-bit slot indices while every index, and the grid stride past the last one, fits
        if (threads + (size_t)g * kThreads * KI_COPY2D_NARROW_INFLIGHT < (1ull << 32))
            vcopy2d_narrow_kernel<uint32_t><<<g, kThreads, 0, ki::as_stream(stream)>>>(a);
        else
            vcopy2d_narrow_kernel<size_t><<<g, kThreads, 0, ki::as_stream(stream)>>>(a);
        return ki::check_launch(ctx, "vcopy2d_narrow_kernel launch");
    }
    vcopy2d_kernel<<<(unsigned)grid_for(ctx, height * a.spans), kThreads, 0, ki::as_stream(stream)>>>(a);
    return ki::check_launch(ctx, "vcopy2d_kernel launch");
}

extern "C" int ki_vcopy_strided(ki_ctx* ctx, void* dst, int64_t dst_stride, const void* src, int64_t src_stride,
                                size_t elem_bytes, size_t count, void* stream) {
    KI_CHECK_CTX(ctx);
    if (count == 0) return KI_OK;
    if (!dst || !src) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_strided: null pointer");
    if (elem_bytes == 0 || elem_bytes > 65536)
        return ki::set_error(ctx, KI_ERR_ARG, "vcopy_strided: element size must be 1 to 65536 bytes");
    size_t word = 16;  // the largest power of two (<= 16) that divides the element size
    while (elem_bytes % word) word >>= 1;
    if (!ki::aligned(dst, word) || !ki::aligned(src, word))
        return ki::set_error(ctx, KI_ERR_ARG,
                             "vcopy_strided: pointers must be aligned to the largest power of two (<= 16) dividing the "
                             "element size");
    const int64_t lim = INT64_MAX / (int64_t)elem_bytes / (int64_t)(count > 0 ? count : 1);
    if (dst_stride > lim || dst_stride < -lim || src_stride > lim || src_stride < -lim)
        return ki::set_error(ctx, KI_ERR_ARG, "vcopy_strided: stride too large");
    if (count > 1 && dst_stride == 0) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_strided: zero destination stride");
    uintptr_t dl, dh, sl, sh;
    span_of((uintptr_t)dst, dst_stride * (int64_t)elem_bytes, count, elem_bytes, &dl, &dh);
    span_of((uintptr_t)src, src_stride * (int64_t)elem_bytes, count, elem_bytes, &sl, &sh);
    if (dl < sh && sl < dh) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_strided: source and destination ranges overlap");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    uint8_t* d = static_cast<uint8_t*>(dst);
    const uint8_t* sp = static_cast<const uint8_t*>(src);
    if (word != elem_bytes) {  // a struct: nw words of `word` bytes per element
        const unsigned nw = (unsigned)(elem_bytes / word);
        if (count > SIZE_MAX / nw) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_strided: too many elements");
        const unsigned g = (unsigned)grid_for(ctx, (count * nw + 31) / 32);
        const int64_t dsb = dst_stride * (int64_t)elem_bytes, ssb = src_stride * (int64_t)elem_bytes;
        switch (word) {
            case 1: strided_words_kernel<1><<<g, kThreads, 0, s>>>(d, dsb, sp, ssb, count, nw); break;
            case 2: strided_words_kernel<2><<<g, kThreads, 0, s>>>(d, dsb, sp, ssb, count, nw); break;
            case 4: strided_words_kernel<4><<<g, kThreads, 0, s>>>(d, dsb, sp, ssb, count, nw); break;
            case 8: strided_words_kernel<8><<<g, kThreads, 0, s>>>(d, dsb, sp, ssb, count, nw); break;
            default: strided_words_kernel<16><<<g, kThreads, 0, s>>>(d, dsb, sp, ssb, count, nw); break;
        }
        return ki::check_launch(ctx, "strided_words_kernel launch");
    }
    const unsigned g = (unsigned)grid_for(ctx, (count + 32 * kUnroll - 1) / (32 * kUnroll));
    switch (elem_bytes) {
        case 1: strided_kernel<1><<<g, kThreads, 0, s>>>(d, dst_stride, sp, src_stride, count); break;
        case 2: strided_kernel<2><<<g, kThreads, 0, s>>>(d, dst_stride, sp, src_stride, count); break;
        case 4: strided_kernel<4><<<g, kThreads, 0, s>>>(d, dst_stride, sp, src_stride, count); break;
        case 8: strided_kernel<8><<<g, kThreads, 0, s>>>(d, dst_stride, sp, src_stride, count); break;
        default: strided_kernel<16><<<g, kThreads, 0, s>>>(d, dst_stride, sp, src_stride, count); break;
    }
    return ki::check_launch(ctx, "strided_kernel launch");
}
