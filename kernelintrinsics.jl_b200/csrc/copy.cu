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
//
// Launches use programmatic dependent launch: a warp prefetches its first span's source words into
// L2 (hints only), then waits for the previous kernel in the stream to complete before it loads or
// stores anything.  Back to back (256 copies of 2^28 bytes) this took the step from 22.7 to 22.2 ms
// (0.923 -> 0.948 of the copy peak): the next copy's dispatch and first reads overlap this one's tail.
#include "ki/bytes.cuh"
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"

namespace {

#ifndef KI_COPY_PDL
#define KI_COPY_PDL 1
#endif
#ifndef KI_COPY_THREADS
#define KI_COPY_THREADS 512
#endif
#ifndef KI_COPY_UNROLL
#define KI_COPY_UNROLL 4
#endif
#ifndef KI_COPY_MIN_BLOCKS
#define KI_COPY_MIN_BLOCKS 1
#endif
#ifndef KI_COPY_WAVES
#define KI_COPY_WAVES 2  // grid = whole waves of resident blocks
#endif
constexpr int kThreads = KI_COPY_THREADS;
constexpr int kUnroll = KI_COPY_UNROLL;  // 32-chunk rows per warp span
constexpr int kSpan = 32 * kUnroll;      // 16-byte chunks per warp span

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
#if KI_COPY_PDL
    {  // programmatic dependent launch: L2 prefetches of this warp's first span (hints), then wait
       // for the previous kernel in the stream to complete before any load or store
        const size_t w0 = ((size_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const size_t k = w0 * kSpan + lane + 32 * j;
            if (k < nc) asm volatile("prefetch.global.L2 [%0];" ::"l"(sa + k));
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
#endif

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
                uint4 hi = ki::shfl_down_u4(lo[j]);
                if (lane == 31) hi = ex[j];
                if (k < nc) d[k] = ki::realign<WS>(lo[j], hi, a.sh);
            }
        }
    }
}

// Resident blocks per SM of one vcopy_kernel instantiation (queried once per context).
template <int WS, bool ALIGNED>
int resident_blocks(ki_ctx* ctx, int idx) {
    if (ctx->copy_resident[idx] == 0) {
        int r = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, vcopy_kernel<WS, ALIGNED>, kThreads, 0) != cudaSuccess ||
            r < 1)
            r = 1;
        ctx->copy_resident[idx] = r;
    }
    return ctx->copy_resident[idx];
}

template <int WS, bool ALIGNED>
int launch_one(ki_ctx* ctx, const CopyArgs& a, size_t want_blocks, int idx, cudaStream_t st) {
    // Whole waves only: a grid that is not a multiple of the resident blocks leaves a partial last
    // wave in which some SMs stream at a fraction of their occupancy.
    const size_t wave = (size_t)ctx->sm_count * resident_blocks<WS, ALIGNED>(ctx, idx);
    size_t blocks = wave * KI_COPY_WAVES;
    if (want_blocks < blocks) blocks = want_blocks;
#if KI_COPY_PDL
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KI_CUDA(ctx, cudaLaunchKernelEx(&cfg, vcopy_kernel<WS, ALIGNED>, a));
    return KI_OK;
#else
    vcopy_kernel<WS, ALIGNED><<<(unsigned)blocks, kThreads, 0, st>>>(a);
    return ki::check_launch(ctx, "vcopy_kernel launch");
#endif
}

// dst, src device pointers that do not overlap; nbytes > 0; device already current.
int launch_vcopy(ki_ctx* ctx, void* dst, const void* src, size_t nbytes, cudaStream_t st) {
    const uintptr_t d0 = (uintptr_t)dst, s0 = (uintptr_t)src;
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
    size_t want = (nspans + (kThreads / 32) - 1) / (kThreads / 32);
    if (want < 1) want = 1;
    if (s == 0) return launch_one<0, true>(ctx, a, want, 0, st);
    if (s < 4) return launch_one<0, false>(ctx, a, want, 1, st);
    if (s < 8) return launch_one<1, false>(ctx, a, want, 2, st);
    if (s < 12) return launch_one<2, false>(ctx, a, want, 3, st);
    return launch_one<3, false>(ctx, a, want, 4, st);
}

}  // namespace

// Streams and events of the host-buffer pipelines (ki_vcopy_host, ki_scan_inclusive_i64_host), made
// on first use.
int ki_ensure_pipe(ki_ctx* ctx) {
    if (ctx->pipe_end) return KI_OK;
    for (int i = 0; i < 3; ++i)
        if (!ctx->pipe_stream[i])
            KI_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->pipe_stream[i], cudaStreamNonBlocking));
    for (int k = 0; k < KI_PIPE_SLOTS; ++k) {
        if (!ctx->pipe_landed[k]) KI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->pipe_landed[k], cudaEventDisableTiming));
        if (!ctx->pipe_copied[k]) KI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->pipe_copied[k], cudaEventDisableTiming));
        if (!ctx->pipe_drained[k])
            KI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->pipe_drained[k], cudaEventDisableTiming));
    }
    if (!ctx->pipe_begin) KI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->pipe_begin, cudaEventDisableTiming));
    KI_CUDA(ctx, cudaEventCreateWithFlags(&ctx->pipe_end, cudaEventDisableTiming));  // last: marks "complete"
    return KI_OK;
}

namespace {

bool overlap(uintptr_t d0, uintptr_t s0, size_t n) { return d0 < s0 + n && s0 < d0 + n; }

}  // namespace

extern "C" int ki_vcopy(ki_ctx* ctx, void* dst, const void* src, size_t nbytes, void* stream) {
    KI_CHECK_CTX(ctx);
    if (nbytes == 0) return KI_OK;
    if (!dst || !src) return ki::set_error(ctx, KI_ERR_ARG, "vcopy: null pointer");
    if (overlap((uintptr_t)dst, (uintptr_t)src, nbytes))
        return ki::set_error(ctx, KI_ERR_ARG, "vcopy: source and destination overlap");
    KI_GUARD(ctx);
    return launch_vcopy(ctx, dst, src, nbytes, ki::as_stream(stream));
}

// Chunks of KI_PIPE_CHUNK bytes go host -> device on stream 0, are copied by vcopy_kernel on
// stream 1 and come back on stream 2, cycling over KI_PIPE_SLOTS staging slots; events order the
// three streams per slot, so both copy directions and the kernel run concurrently.  Inside each
// slot a chunk keeps its host address modulo 16, so the kernel sees the caller's misalignment.
extern "C" int ki_vcopy_host(ki_ctx* ctx, void* dst, const void* src, size_t nbytes, void* stream) {
    KI_CHECK_CTX(ctx);
    if (nbytes == 0) return KI_OK;
    if (!dst || !src) return ki::set_error(ctx, KI_ERR_ARG, "vcopy_host: null pointer");
    if (overlap((uintptr_t)dst, (uintptr_t)src, nbytes))
        return ki::set_error(ctx, KI_ERR_ARG, "vcopy_host: source and destination overlap");
    KI_GUARD(ctx);
    int rc = ki_ensure_pipe(ctx);
    if (rc) return rc;
    constexpr size_t kChunk = KI_PIPE_CHUNK;
    constexpr size_t kSlot = kChunk + 256;
    void* stage = nullptr;
    rc = ki::ensure_region(ctx, KI_REG_STAGE, 2 * KI_PIPE_SLOTS * kSlot, &stage);
    if (rc) return rc;
    cudaStream_t s = ki::as_stream(stream);
    cudaStream_t up = ctx->pipe_stream[0], kern = ctx->pipe_stream[1], down = ctx->pipe_stream[2];
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_begin, s));
    for (int i = 0; i < 3; ++i) KI_CUDA(ctx, cudaStreamWaitEvent(ctx->pipe_stream[i], ctx->pipe_begin, 0));
    const size_t so = (uintptr_t)src & 15, dso = (uintptr_t)dst & 15;
    const uint8_t* hs = static_cast<const uint8_t*>(src);
    uint8_t* hd = static_cast<uint8_t*>(dst);
    uint8_t* base = static_cast<uint8_t*>(stage);
    const size_t nch = (nbytes + kChunk - 1) / kChunk;
    for (size_t i = 0; i < nch; ++i) {
        const int k = (int)(i % KI_PIPE_SLOTS);
        const size_t off = i * kChunk, len = (nbytes - off < kChunk) ? nbytes - off : kChunk;
        uint8_t* in = base + (size_t)k * kSlot + so;
        uint8_t* out = base + (size_t)(KI_PIPE_SLOTS + k) * kSlot + dso;
        if (i >= (size_t)KI_PIPE_SLOTS) {
            KI_CUDA(ctx, cudaStreamWaitEvent(up, ctx->pipe_copied[k], 0));     // input slot read
            KI_CUDA(ctx, cudaStreamWaitEvent(kern, ctx->pipe_drained[k], 0));  // output slot sent back
        }
        KI_CUDA(ctx, cudaMemcpyAsync(in, hs + off, len, cudaMemcpyHostToDevice, up));
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_landed[k], up));
        KI_CUDA(ctx, cudaStreamWaitEvent(kern, ctx->pipe_landed[k], 0));
        rc = launch_vcopy(ctx, out, in, len, kern);
        if (rc) return rc;
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_copied[k], kern));
        KI_CUDA(ctx, cudaStreamWaitEvent(down, ctx->pipe_copied[k], 0));
        KI_CUDA(ctx, cudaMemcpyAsync(hd + off, out, len, cudaMemcpyDeviceToHost, down));
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_drained[k], down));
    }
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_end, down));
    KI_CUDA(ctx, cudaStreamWaitEvent(s, ctx->pipe_end, 0));
    return KI_OK;
}
