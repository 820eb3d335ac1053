// scan.cu -- single-pass decoupled-lookback inclusive scan of Int64 (Base.cumsum semantics).
//
// One persistent CTA per SM, software-pipelined over tiles of 15872 elements, with 31 "work" warps
// and one "look" warp (1024 threads).  Iteration k of a CTA runs two phases:
//   phase A  work warps: wait for tile k (one 124 KiB 1-D TMA bulk copy, cp.async.bulk ...
//            mbarrier::complete_tx), sum it (warp w folds its 512 elements with @warpfold over 8 rows
//            of 32 lanes x 2 elements; warp 0 scans the 31 warp totals with @warpreduce) and publish
//            its aggregate at once (ki/lookback.cuh: packed 64-bit status word, st.release.gpu);
//            look warp, at the same time: the decoupled lookback of tile k-1;
//   phase B  the look warp takes the next ticket and starts its TMA into the (now free) tile buffer;
//            work warps finish tile k-1: re-read its span from global memory (still in the 126 MB
//            L2), rescan each row with @warpreduce (src/warp.jl:226-237) from the running prefix and
//            store it with coalesced 16-byte streaming stores.
// Between taking a ticket and publishing that tile's aggregate a CTA only waits for its own load and
// its own second pass, never for a lookback, so no aggregate waits behind another tile; and the
// ~1 us L2 round trips of a lookback overlap the next tile's load and first pass.  Tile indices
// come from an atomic ticket, so a tile's predecessors are always taken by CTAs that already run.
// Tiles that are partial or not 16-byte aligned are staged with plain loads.
//
// Why one large CTA per SM: a lookback costs L2 round trips in proportion to the number of tiles
// in flight ahead of it, and a tile's bytes set how long its CTA has before the next one; few, large
// tiles keep the lookback inside the pipeline, and 30 warps keep enough loads in flight.  Measured
// at n = 2^30: 4096-element tiles x 3 CTAs/SM 0.78 of HBM peak, 8192 x 2 0.82, 12288 x 1 (24 warps)
// 0.88, 15360 x 1 (30 warps) 0.92, 15872 x 1 (31 warps) 0.94.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"

// Tiles are read twice: once by TMA for the first pass, once from L2 for the second.
#ifndef KI_KEEP_TILES
#define KI_KEEP_TILES 1
#endif
#if KI_KEEP_TILES
#define KI_G2S ki::bulk_g2s_keep
#define KI_RELOAD(p) __ldcs(p)
#else
#define KI_G2S ki::bulk_g2s
#define KI_RELOAD(p) (*(p))
#endif

namespace {

#ifndef KI_SCAN_TILE
#define KI_SCAN_TILE 15872
#endif
#ifndef KI_SCAN_WORK_WARPS
#define KI_SCAN_WORK_WARPS 31
#endif
constexpr int kWorkWarps = KI_SCAN_WORK_WARPS;
constexpr int kLookWarp = kWorkWarps;
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = kWorkThreads + 32;
constexpr int kTile = KI_SCAN_TILE;             // elements per tile
constexpr int kWarpSpan = kTile / kWorkWarps;   // elements per work warp (512)
constexpr int kRows = kWarpSpan / 64;           // rows of 32 lanes x 2 elements
static_assert(kWarpSpan % 64 == 0 && kWorkWarps <= 32, "tile must split into rows of 64 elements per warp");
constexpr int kBatch = kRows < 8 ? kRows : 8;   // rows loaded at once in the second pass
constexpr size_t kSmemBytes = kTile * sizeof(int64_t);
#ifndef KI_SCAN_LOOKBACK_K
#define KI_SCAN_LOOKBACK_K 1
#endif
#ifndef KI_SCAN_CTAS_PER_SM
#define KI_SCAN_CTAS_PER_SM 1
#endif
constexpr int kLookbackK = KI_SCAN_LOOKBACK_K;  // lookback window of 32*K tiles per round trip
constexpr int kCtasPerSm = KI_SCAN_CTAS_PER_SM;

struct ScanArgs {
    const int64_t* in;
    int64_t* out;
    size_t n;
    int64_t seed;
    const int64_t* seed_ptr;  // when set, the seed is read from device memory at the start
    ki::TileStatus st;
    unsigned long long* ticket;
    uint32_t* status;
    uint64_t timeout_ns;
    int tma_in;   // input 16-byte aligned: full tiles come in by TMA
    int vec_out;  // output 16-byte aligned: full tiles leave with 16-byte stores
};

struct Pending {
    unsigned long long t;
    int64_t agg;
    int64_t tile_excl;
    int64_t warp_excl[kWorkWarps];
};

__device__ __forceinline__ void work_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkThreads) : "memory"); }

__global__ void __launch_bounds__(kThreads) scan_i64_kernel(ScanArgs a) {
    // every CTA of this persistent grid is resident from the start, so a dependent kernel launched
    // with programmatic stream serialization (a sharded scan's next phase-1 reduce) may be
    // dispatched as CTAs retire; it waits for this kernel to complete before touching memory
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    int64_t* sb = reinterpret_cast<int64_t*>(smem_raw);
    __shared__ __align__(8) uint64_t bar;
    __shared__ int64_t warp_tot[kWorkWarps];
    __shared__ Pending slot[2];  // tile k (being summed) and tile k-1 (being finished)
    __shared__ unsigned long long ticket;

    const int tid = threadIdx.x;
    const int w = tid >> 5;
    const unsigned lane = tid & 31;
    const uint64_t ntiles = (a.n + kTile - 1) / kTile;
    // only tile 0 uses the seed (its inclusive prefix is seed + aggregate; lookbacks stop there)
    const int64_t seed = a.seed_ptr ? *a.seed_ptr : a.seed;
    auto bulk_ok = [&](uint64_t t) { return a.tma_in && t < ntiles && (t + 1) * (uint64_t)kTile <= a.n; };
    auto fetch = [&]() {  // take a ticket and start its load (one thread)
        const unsigned long long t = atomicAdd(a.ticket, 1ull);
        ticket = t;
        if (bulk_ok(t)) {
            ki::fence_proxy_async_smem();  // earlier generic reads of sb come first
            ki::mbar_arrive_expect_tx(&bar, (uint32_t)kSmemBytes);
            KI_G2S(sb, a.in + t * kTile, (uint32_t)kSmemBytes, &bar);
        }
    };
    if (tid == 0) {
        ki::mbar_init(&bar, 1);
        ki::fence_mbar_init();
        fetch();
    }
    __syncthreads();

    uint32_t phase = 0;
    bool have_old = false;
    int cur = 0;  // slot of tile k; tile k-1 is in slot cur ^ 1
    while (true) {
        const uint64_t t_new = ticket;
        const bool new_valid = t_new < ntiles;
        if (!new_valid && !have_old) break;

        // ---- phase A: sum and publish tile k  ||  look back for tile k-1 ---------------------------
        if (w == kLookWarp) {
            if (have_old) {
                Pending& o = slot[cur ^ 1];
                const int64_t ex = ki::decoupled_lookback<kLookbackK>(a.st, o.t, o.agg, seed, a.status,
                                                                      a.timeout_ns);
                if (lane == 0) o.tile_excl = ex;
            }
        } else if (new_valid) {
            const size_t first = (size_t)t_new * kTile;
            const int count = (int)min((size_t)kTile, a.n - first);
            if (bulk_ok(t_new)) {
                if (!ki::mbar_wait_bounded(&bar, phase, a.status, a.timeout_ns))
                    ki::mbar_wait_bounded(&bar, phase, a.status, a.timeout_ns);  // never leave a copy in flight
                phase ^= 1u;
            } else {
                for (int i = tid; i < kTile; i += kWorkThreads) sb[i] = (i < count) ? a.in[first + i] : 0;
                work_sync();
            }
            int64_t s = 0;
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                const longlong2 p = *reinterpret_cast<const longlong2*>(sb + w * kWarpSpan + 64 * j + 2 * lane);
                s = ki::wrap_add(s, ki::wrap_add(p.x, p.y));
            }
            s = ki::warpfold(s, ki::WrapAdd{});
            if (lane == 0) warp_tot[w] = s;
            work_sync();
            if (w == 0) {
                const int64_t x = (lane < (unsigned)kWorkWarps) ? warp_tot[lane] : 0;
                const int64_t inc = ki::warpreduce(x, ki::WrapAdd{});
                const int64_t agg = __shfl_sync(0xffffffffu, inc, kWorkWarps - 1);
                Pending& e = slot[cur];
                if (lane < (unsigned)kWorkWarps) e.warp_excl[lane] = ki::wrap_sub(inc, x);
                if (lane == 0) {
                    e.t = t_new;
                    e.agg = agg;
                    ki::publish_aggregate(a.st, t_new, agg, seed);
                }
            }
        }
        __syncthreads();  // tile k summed (buffer free, slot written); tile k-1's prefix known

        // ---- phase B: start tile k+1's load; finish tile k-1 ------------------------------------------
        if (tid == kLookWarp * 32 && new_valid) fetch();  // the look warp is idle in phase B
        if (w < kWorkWarps && have_old) {
            const Pending& o = slot[cur ^ 1];
            const size_t first = (size_t)o.t * kTile;
            const int count = (int)min((size_t)kTile, a.n - first);
            const bool full = count == kTile;
            int64_t carry = ki::wrap_add(o.tile_excl, o.warp_excl[w]);
#pragma unroll
            for (int j0 = 0; j0 < kRows; j0 += kBatch) {
                longlong2 v[kBatch];
#pragma unroll
                for (int jj = 0; jj < kBatch; ++jj) {  // a batch of loads in flight before the scan
                    const int i = w * kWarpSpan + 64 * (j0 + jj) + 2 * (int)lane;
                    if (full && a.tma_in) {
                        v[jj] = KI_RELOAD(reinterpret_cast<const longlong2*>(a.in + first + i));
                    } else {
                        v[jj].x = (i < count) ? a.in[first + i] : 0;
                        v[jj].y = (i + 1 < count) ? a.in[first + i + 1] : 0;
                    }
                }
#pragma unroll
                for (int jj = 0; jj < kBatch; ++jj) {
                    const int64_t pair = ki::wrap_add(v[jj].x, v[jj].y);
                    const int64_t inc = ki::warpreduce(pair, ki::WrapAdd{});
                    const int64_t o0 = ki::wrap_add(ki::wrap_add(carry, ki::wrap_sub(inc, pair)), v[jj].x);
                    const int64_t o1 = ki::wrap_add(o0, v[jj].y);
                    const int i = w * kWarpSpan + 64 * (j0 + jj) + 2 * (int)lane;
                    if (full && a.vec_out) {
                        __stcs(reinterpret_cast<longlong2*>(a.out + first + i), make_longlong2(o0, o1));
                    } else {
                        if (i < count) a.out[first + i] = o0;
                        if (i + 1 < count) a.out[first + i + 1] = o1;
                    }
                    carry = ki::wrap_add(carry, __shfl_sync(0xffffffffu, inc, 31));
                }
            }
        }
        __syncthreads();  // the next ticket is visible; slot cur ^ 1 is free
        have_old = new_valid;
        cur ^= 1;
    }
}

// Grid and launch shared by both entry points: persistent, kCtasPerSm CTAs per SM.
void launch_scan(const ScanArgs& a, size_t ntiles, int sm_count, cudaStream_t s) {
    size_t grid = (size_t)sm_count * kCtasPerSm;
    if (grid > ntiles) grid = ntiles;
    scan_i64_kernel<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(a);
}

}  // namespace

namespace {

int scan_i64_ctx(ki_ctx* ctx, const int64_t* d_in, int64_t* d_out, size_t n, int64_t seed, const int64_t* d_seed,
                 cudaStream_t s) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_in || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "scan: null pointer");
    if (!ki::aligned(d_in, 8) || !ki::aligned(d_out, 8))
        return ki::set_error(ctx, KI_ERR_ARG, "scan: Int64 pointers must be 8-byte aligned");
    if (d_seed && !ki::aligned(d_seed, 8)) return ki::set_error(ctx, KI_ERR_ARG, "scan: misaligned seed");
    if (d_in != d_out) {
        const uintptr_t i0 = (uintptr_t)d_in, o0 = (uintptr_t)d_out, nb = n * sizeof(int64_t);
        if (i0 < o0 + nb && o0 < i0 + nb)
            return ki::set_error(ctx, KI_ERR_ARG, "scan: partially overlapping input and output");
    }
    KI_GUARD(ctx);
    const size_t ntiles = (n + kTile - 1) / kTile;
    if (ntiles > (size_t)INT32_MAX) return ki::set_error(ctx, KI_ERR_ARG, "scan: n too large");
    // scratch: [ticket (256 B)] [status words ntiles] [aggs ntiles] [incls ntiles]
    const size_t words_off = 256;
    const size_t bytes = words_off + ntiles * 24;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_SCAN, bytes, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, words_off + ntiles * sizeof(uint64_t), s));

    KI_CUDA(ctx, cudaFuncSetAttribute(scan_i64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSmemBytes));
    ScanArgs a;
    a.in = d_in;
    a.out = d_out;
    a.n = n;
    a.seed = seed;
    a.seed_ptr = d_seed;
    a.st.words = reinterpret_cast<uint64_t*>(b + words_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + words_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + words_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.tma_in = ki::aligned(d_in, 16);
    a.vec_out = ki::aligned(d_out, 16);
    launch_scan(a, ntiles, ctx->sm_count, s);
    return ki::check_launch(ctx, "scan_i64_kernel launch");
}

}  // namespace

extern "C" int ki_scan_inclusive_i64(ki_ctx* ctx, const int64_t* d_in, int64_t* d_out, size_t n, int64_t seed,
                                     void* stream) {
    return scan_i64_ctx(ctx, d_in, d_out, n, seed, nullptr, ki::as_stream(stream));
}

// Everything a scan of up to n elements needs before it can be enqueued without a blocking call:
// the tile-status scratch (cudaMalloc on first use or growth) and the kernel's shared-memory
// attribute (which also loads the kernel under lazy module loading).  Sharded scans call this before
// their exchange: a cudaMalloc or a module load issued after it could wait for a device whose
// exchange kernel waits for a rank that the same host thread has not reached yet.
__attribute__((visibility("hidden"))) int ki_scan_i64_reserve(ki_ctx* ctx, size_t n) {
    const size_t ntiles = (n + kTile - 1) / kTile;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_SCAN, 256 + ntiles * 24, &base);
    if (rc) return rc;
    KI_CUDA(ctx, cudaFuncSetAttribute(scan_i64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    return KI_OK;
}

extern "C" int ki_scan_inclusive_i64_dseed(ki_ctx* ctx, const int64_t* d_in, int64_t* d_out, size_t n,
                                           const int64_t* d_seed, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_seed) return ki::set_error(ctx, KI_ERR_ARG, "scan: null seed pointer");
    return scan_i64_ctx(ctx, d_in, d_out, n, 0, d_seed, ki::as_stream(stream));
}

// Inclusive scan of HOST buffers through the device.  Chunks of KI_PIPE_CHUNK bytes go host ->
// device on pipe stream 0, are scanned on stream 1 and come back on stream 2, cycling over
// KI_PIPE_SLOTS staging slots (the pipeline of ki_vcopy_host), so both copy directions and the scans
// overlap.  Chunk i > 0 is seeded on the device with the last output of chunk i-1, which is still in
// its staging slot: that slot is rewritten only by chunk i-1+KI_PIPE_SLOTS, whose scan runs after
// chunk i's on the same stream.
extern "C" int ki_scan_inclusive_i64_host(ki_ctx* ctx, const int64_t* h_in, int64_t* h_out, size_t n, int64_t seed,
                                          void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!h_in || !h_out) return ki::set_error(ctx, KI_ERR_ARG, "scan_host: null pointer");
    if (!ki::aligned(h_in, 8) || !ki::aligned(h_out, 8))
        return ki::set_error(ctx, KI_ERR_ARG, "scan_host: Int64 pointers must be 8-byte aligned");
    if (h_in != h_out) {
        const uintptr_t i0 = (uintptr_t)h_in, o0 = (uintptr_t)h_out, nb = n * sizeof(int64_t);
        if (i0 < o0 + nb && o0 < i0 + nb)
            return ki::set_error(ctx, KI_ERR_ARG, "scan_host: partially overlapping input and output");
    }
    KI_GUARD(ctx);
    int rc = ki_ensure_pipe(ctx);
    if (rc) return rc;
    constexpr size_t kChunk = KI_PIPE_CHUNK / sizeof(int64_t);  // elements per chunk
    void* stage = nullptr;
    rc = ki::ensure_region(ctx, KI_REG_STAGE, 2 * KI_PIPE_SLOTS * (size_t)KI_PIPE_CHUNK, &stage);
    if (rc) return rc;
    int64_t* base = static_cast<int64_t*>(stage);
    cudaStream_t s = ki::as_stream(stream);
    cudaStream_t up = ctx->pipe_stream[0], kern = ctx->pipe_stream[1], down = ctx->pipe_stream[2];
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_begin, s));
    for (int i = 0; i < 3; ++i) KI_CUDA(ctx, cudaStreamWaitEvent(ctx->pipe_stream[i], ctx->pipe_begin, 0));
    const size_t nch = (n + kChunk - 1) / kChunk;
    const int64_t* prev_last = nullptr;
    for (size_t i = 0; i < nch; ++i) {
        const int k = (int)(i % KI_PIPE_SLOTS);
        const size_t off = i * kChunk, len = (n - off < kChunk) ? n - off : kChunk;
        int64_t* in = base + (size_t)k * kChunk;
        int64_t* out = base + (size_t)(KI_PIPE_SLOTS + k) * kChunk;
        if (i >= (size_t)KI_PIPE_SLOTS) {
            KI_CUDA(ctx, cudaStreamWaitEvent(up, ctx->pipe_copied[k], 0));     // input slot read
            KI_CUDA(ctx, cudaStreamWaitEvent(kern, ctx->pipe_drained[k], 0));  // output slot sent back
        }
        KI_CUDA(ctx, cudaMemcpyAsync(in, h_in + off, len * sizeof(int64_t), cudaMemcpyHostToDevice, up));
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_landed[k], up));
        KI_CUDA(ctx, cudaStreamWaitEvent(kern, ctx->pipe_landed[k], 0));
        rc = scan_i64_ctx(ctx, in, out, len, seed, prev_last, kern);
        if (rc) return rc;
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_copied[k], kern));
        KI_CUDA(ctx, cudaStreamWaitEvent(down, ctx->pipe_copied[k], 0));
        KI_CUDA(ctx, cudaMemcpyAsync(h_out + off, out, len * sizeof(int64_t), cudaMemcpyDeviceToHost, down));
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_drained[k], down));
        prev_last = out + len - 1;
    }
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_end, down));
    KI_CUDA(ctx, cudaStreamWaitEvent(s, ctx->pipe_end, 0));
    return KI_OK;
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc: hosts whose device memory is owned by another allocator (a
// Julia or Python pool that must not be bypassed or grown behind its back), real-time loops that
// forbid allocation after start-up, and code that must not stall the device, as cudaMalloc may.
// ki_scan_inclusive_i64_noalloc runs the same kernel as ki_scan_inclusive_i64 but takes its
// tile-status scratch from the file-scope array below instead of a context, so it needs no context
// and allocates nothing.
//
// The array is sized for KI_SCAN_NOALLOC_MAX_N elements (a 256-byte header plus three 8-byte words
// per tile: 16,913 tiles of 15872 elements, about 397 KiB).  Every GPU that loads this library
// holds it until the process exits.
//
// In host code the array's name is only a host-side stand-in, so its device address is looked up
// with cudaGetSymbolAddress (with the caller's device current) and cached.  A __device__ array's
// address belongs to a CUDA context, not to a device, so the cache is keyed by the unique ID of the
// calling thread's current context (cuCtxGetId): a call from a context not seen before (another
// device, a non-primary context, a primary context re-created after cudaDeviceReset) repeats the
// set-up.  The set-up runs, once per context: cudaGetSymbolAddress (which also loads the module
// under lazy loading), cudaDeviceGetAttribute (SM count) and cudaFuncSetAttribute (dynamic shared
// memory).  Every call also runs cuCtxGetCurrent and cuCtxGetId, reached through
// cudaGetDriverEntryPointByVersion so the library does not link libcuda; when no context is current
// it first runs cudaGetDevice and cudaSetDevice, which bind the device's primary context.  Make the
// first call in each context before any stream capture.
//
// All calls share the array and it keeps the last call's contents: each call clears the ticket, the
// status word and the tile status words (cudaMemsetAsync on the cached address) before its launch,
// and calls that overlap on the GPU (different streams, or several host threads) race on it.
// A bounded wait that runs out is latched in the array's status word and not reported; use the
// context API where timeout reporting is needed.
// ---------------------------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocTiles = (KI_SCAN_NOALLOC_MAX_N + kTile - 1) / kTile;
constexpr size_t kNoAllocHeader = 256;  // ticket at 0, status word at 64
static __device__ __align__(256) unsigned char g_scan_noalloc_scratch[kNoAllocHeader + kNoAllocTiles * 24];

struct NoAllocContext {
    unsigned long long ctx_id = 0;  // cuCtxGetId of the context the address belongs to (0: free slot)
    unsigned char* scratch = nullptr;
    int sm_count = 0;
};
constexpr int kNoAllocContexts = 64;
std::mutex g_noalloc_mutex;
NoAllocContext g_noalloc_ctx[kNoAllocContexts];
int g_noalloc_next = 0;  // slot taken by the next new context (round robin once all are used)

typedef int (*CtxGetCurrentFn)(void** ctx);                   // cuCtxGetCurrent
typedef int (*CtxGetIdFn)(void* ctx, unsigned long long* id);  // cuCtxGetId
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

// Unique ID of the calling thread's current CUDA context, 0 on failure.  Called with the mutex held.
unsigned long long current_context_id() {
    if (!g_ctx_get_current || !g_ctx_get_id) {
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f1, 12000, cudaEnableDefault, &q1) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess || !f1)
            return 0;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f2, 12000, cudaEnableDefault, &q2) != cudaSuccess ||
            q2 != cudaDriverEntryPointSuccess || !f2)
            return 0;
        g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
        g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
    void* c = nullptr;
    unsigned long long id = 0;
    if (g_ctx_get_current(&c) != 0) return 0;
    if (!c) {  // no context current yet: cudaSetDevice initialises and binds the device's primary context
        int dev = -1;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return 0;
        if (g_ctx_get_current(&c) != 0 || !c) return 0;
    }
    if (g_ctx_get_id(c, &id) != 0) return 0;
    return id;
}

}  // namespace

extern "C" int ki_scan_inclusive_i64_noalloc(const int64_t* d_in, int64_t* d_out, size_t n, int64_t seed,
                                             void* stream) {
    if (n == 0) return KI_OK;
    if (n > (size_t)KI_SCAN_NOALLOC_MAX_N) return KI_ERR_ARG;  // beyond the static scratch
    if (!d_in || !d_out) return KI_ERR_ARG;
    if (!ki::aligned(d_in, 8) || !ki::aligned(d_out, 8)) return KI_ERR_ARG;
    if (d_in != d_out) {
        const uintptr_t i0 = (uintptr_t)d_in, o0 = (uintptr_t)d_out, nb = n * sizeof(int64_t);
        if (i0 < o0 + nb && o0 < i0 + nb) return KI_ERR_ARG;
    }
    unsigned char* scratch = nullptr;
    int sm_count = 0;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        const unsigned long long id = current_context_id();
        if (id == 0) return KI_ERR_CUDA;
        NoAllocContext* c = nullptr;
        for (auto& e : g_noalloc_ctx)
            if (e.ctx_id == id) c = &e;
        if (!c) {  // first call in this context: look the array up and prepare the kernel
            int dev = -1, sms = 0;
            void* p = nullptr;
            if (cudaGetDevice(&dev) != cudaSuccess) return KI_ERR_CUDA;
            if (cudaGetSymbolAddress(&p, g_scan_noalloc_scratch) != cudaSuccess || !p) return KI_ERR_CUDA;
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
                return KI_ERR_CUDA;
            if (cudaFuncSetAttribute(scan_i64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSmemBytes) != cudaSuccess)
                return KI_ERR_CUDA;
            c = &g_noalloc_ctx[g_noalloc_next];
            g_noalloc_next = (g_noalloc_next + 1) % kNoAllocContexts;
            c->ctx_id = id;
            c->scratch = static_cast<unsigned char*>(p);
            c->sm_count = sms;
        }
        scratch = c->scratch;
        sm_count = c->sm_count;
    }
    const size_t ntiles = (n + kTile - 1) / kTile;
    cudaStream_t s = ki::as_stream(stream);
    if (cudaMemsetAsync(scratch, 0, kNoAllocHeader + ntiles * sizeof(uint64_t), s) != cudaSuccess)
        return KI_ERR_CUDA;
    ScanArgs a;
    a.in = d_in;
    a.out = d_out;
    a.n = n;
    a.seed = seed;
    a.seed_ptr = nullptr;
    a.st.words = reinterpret_cast<uint64_t*>(scratch + kNoAllocHeader);
    a.st.aggs = reinterpret_cast<int64_t*>(scratch + kNoAllocHeader + kNoAllocTiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(scratch + kNoAllocHeader + kNoAllocTiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(scratch);
    a.status = reinterpret_cast<uint32_t*>(scratch + 64);
    a.timeout_ns = 2000000000ull;
    a.tma_in = ki::aligned(d_in, 16);
    a.vec_out = ki::aligned(d_out, 16);
    // cudaLaunchKernel returns this launch's own status: an earlier, unrelated error left in the
    // runtime's last-error slot is neither returned nor cleared.
    size_t grid = (size_t)sm_count * kCtasPerSm;
    if (grid > ntiles) grid = ntiles;
    void* args[] = {&a};
    const cudaError_t e =
        cudaLaunchKernel((const void*)scan_i64_kernel, dim3((unsigned)grid), dim3(kThreads), args, kSmemBytes, s);
    return e == cudaSuccess ? KI_OK : KI_ERR_CUDA;
}
