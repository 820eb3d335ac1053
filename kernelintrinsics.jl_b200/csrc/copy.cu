// copy.cu -- vectorised byte copy (copyto!) at any source / destination alignment.
//
// The reference's vload_multi / vstore_multi! (src/vectorization.jl:306-420) split an N-element
// access at a misaligned address into naturally aligned pieces of at most N/2 elements.  A
// device-wide copy on B200 does better: the destination is split into an unaligned head (< 16 B),
// a 16-byte aligned body and a tail (< 16 B).  Every body store is a full st.global.v4.  When the
// source is misaligned relative to the destination by s bytes, every body load is still an aligned
// ld.global.v4: lane l of a warp loads aligned source word k, takes word k+1 from lane l+1 with
// __shfl_down_sync (lane 31 loads it itself), and funnel-shifts the pair into the 16 output bytes.
// The word shift s/4 is a template parameter; the byte shift (s%4)*8 goes to __funnelshift_r.
//
// Reads of the aligned source words never leave the 16-byte words that hold source bytes, so they
// stay inside the source allocation's pages.  Head and tail bytes are copied by block 0, warp 0.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"

namespace {

#ifndef KI_COPY_THREADS
#define KI_COPY_THREADS 512
#endif
#ifndef KI_COPY_UNROLL
#define KI_COPY_UNROLL 4
#endif
#ifndef KI_COPY_BLOCKS_PER_SM
#define KI_COPY_BLOCKS_PER_SM 4
#endif
#ifndef KI_COPY_MIN_BLOCKS
#define KI_COPY_MIN_BLOCKS 1
#endif
constexpr int kThreads = KI_COPY_THREADS;
constexpr int kUnroll = KI_COPY_UNROLL;  // 32-chunk rows per warp span
constexpr int kSpan = 32 * kUnroll;      // 16-byte chunks per warp span
constexpr int kBlocksPerSm = KI_COPY_BLOCKS_PER_SM;

template <int WS>
__device__ __forceinline__ uint4 realign(const uint4& lo, const uint4& hi, unsigned sh) {
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint4 r;
    r.x = __funnelshift_r(w[WS + 0], w[WS + 1], sh);
    r.y = __funnelshift_r(w[WS + 1], w[WS + 2], sh);
    r.z = __funnelshift_r(w[WS + 2], w[WS + 3], sh);
    r.w = __funnelshift_r(w[WS + 3], w[WS + 4], sh);
    return r;
}

__device__ __forceinline__ uint4 shfl_down_u4(const uint4& v) {
    uint4 r;
    r.x = __shfl_down_sync(0xffffffffu, v.x, 1);
    r.y = __shfl_down_sync(0xffffffffu, v.y, 1);
    r.z = __shfl_down_sync(0xffffffffu, v.z, 1);
    r.w = __shfl_down_sync(0xffffffffu, v.w, 1);
    return r;
}

struct CopyArgs {
    uint8_t* dst;          // start of the whole destination range
    const uint8_t* src;    // start of the whole source range
    size_t head;           // bytes before the 16-byte aligned destination body
    size_t nchunks;        // 16-byte body chunks
    size_t tail;           // bytes after the body
    const uint4* src_al;   // aligned-down source address of the first body byte
    unsigned sh;           // (source misalignment % 4) * 8
};

// WS = source misalignment / 4 within a 16-byte word; ALIGNED when the misalignment is 0.
template <int WS, bool ALIGNED>
__global__ void __launch_bounds__(kThreads, KI_COPY_MIN_BLOCKS) vcopy_kernel(CopyArgs a) {
    const unsigned lane = threadIdx.x & 31;
    uint4* __restrict__ d = reinterpret_cast<uint4*>(a.dst + a.head);
    const uint4* __restrict__ sa = a.src_al;
    const size_t nc = a.nchunks;

    if (blockIdx.x == 0 && threadIdx.x < 32) {
        if (lane < a.head) a.dst[lane] = a.src[lane];
        const size_t t0 = a.head + nc * 16;
        if (lane >= 16 && lane - 16 < a.tail) a.dst[t0 + lane - 16] = a.src[t0 + lane - 16];
    }

    const size_t warp = ((size_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const size_t nwarps = ((size_t)gridDim.x * kThreads) >> 5;
    const size_t nspans = (nc + kSpan - 1) / kSpan;
    for (size_t sp = warp; sp < nspans; sp += nwarps) {
        const size_t base = sp * kSpan + lane;
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
                if (k <= nc) lo[j] = sa[k];                       // word nc still holds source bytes
                if (lane == 31 && k < nc) ex[j] = sa[k + 1];
            }
#pragma unroll
            for (int j = 0; j < kUnroll; ++j) {
                const size_t k = base + 32 * j;
                uint4 hi = shfl_down_u4(lo[j]);
                if (lane == 31) hi = ex[j];
                if (k < nc) d[k] = realign<WS>(lo[j], hi, a.sh);
            }
        }
    }
}

}  // namespace

extern "C" int ki_vcopy(ki_ctx* ctx, void* dst, const void* src, size_t nbytes, void* stream) {
    KI_CHECK_CTX(ctx);
    if (nbytes == 0) return KI_OK;
    if (!dst || !src) return ki::set_error(ctx, KI_ERR_ARG, "vcopy: null pointer");
    const uintptr_t d0 = (uintptr_t)dst, s0 = (uintptr_t)src;
    if (d0 < s0 + nbytes && s0 < d0 + nbytes)
        return ki::set_error(ctx, KI_ERR_ARG, "vcopy: source and destination overlap");
    KI_GUARD(ctx);
    CopyArgs a;
    a.dst = static_cast<uint8_t*>(dst);
    a.src = static_cast<const uint8_t*>(src);
    a.head = (16 - (d0 & 15)) & 15;
    if (a.head > nbytes) a.head = nbytes;
    a.nchunks = (nbytes - a.head) / 16;
    a.tail = nbytes - a.head - a.nchunks * 16;
    const uintptr_t sb = s0 + a.head;
    const unsigned s = (unsigned)(sb & 15);
    a.src_al = reinterpret_cast<const uint4*>(sb - s);
    a.sh = (s & 3) * 8;
    const size_t nspans = (a.nchunks + kSpan - 1) / kSpan;
    size_t blocks = (nspans + (kThreads / 32) - 1) / (kThreads / 32);
    const size_t max_blocks = (size_t)ctx->sm_count * kBlocksPerSm;
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    cudaStream_t st = ki::as_stream(stream);
    const dim3 g((unsigned)blocks), b(kThreads);
    if (s == 0) vcopy_kernel<0, true><<<g, b, 0, st>>>(a);
    else if (s < 4) vcopy_kernel<0, false><<<g, b, 0, st>>>(a);
    else if (s < 8) vcopy_kernel<1, false><<<g, b, 0, st>>>(a);
    else if (s < 12) vcopy_kernel<2, false><<<g, b, 0, st>>>(a);
    else vcopy_kernel<3, false><<<g, b, 0, st>>>(a);
    return ki::check_launch(ctx, "vcopy_kernel launch");
}
