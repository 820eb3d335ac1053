// scan.cu -- single-pass decoupled-lookback inclusive scan of Int64 (Base.cumsum semantics).
//
// One CTA per 4096-element tile (32 KiB), tiles handed out by an atomic ticket so that a tile's
// predecessors are always owned by CTAs that already run (no deadlock on non-resident CTAs).
// A full, 16-byte aligned tile is staged into shared memory with one 1-D TMA bulk copy
// (cp.async.bulk ... mbarrier::complete_tx) and written back with one bulk store.
//
// Inside a tile, warp w owns elements [512w, 512w+512); lane l reads the pairs at 64j+2l (one
// conflict-free 16-byte shared load per j).  Pass 1 folds each warp's 512 elements (xor fold,
// @warpfold with every lane holding the total), warp 0 scans the 8 warp totals with @warpreduce,
// publishes the tile aggregate and runs the decoupled lookback (ki/lookback.cuh) with
// st.release.gpu / ld.acquire.gpu flags.  Pass 2 rescans each pair row with @warpreduce
// (src/warp.jl:226-237) carrying the running prefix.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 4096;                 // elements per tile
constexpr int kWarpSpan = kTile / kWarps;   // 512 elements per warp
constexpr int kRows = kWarpSpan / 64;       // 8 rows of 32 lanes x 2 elements
constexpr size_t kSmemBytes = kTile * sizeof(int64_t);

struct ScanArgs {
    const int64_t* in;
    int64_t* out;
    size_t n;
    int64_t seed;
    ki::TileStatus st;
    unsigned long long* ticket;
    uint32_t* status;
    uint64_t timeout_ns;
    int use_tma;
};

__global__ void __launch_bounds__(kThreads) scan_i64_kernel(ScanArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    int64_t* tile = reinterpret_cast<int64_t*>(smem_raw);
    __shared__ __align__(8) uint64_t bar;
    __shared__ int64_t warp_tot[kWarps];
    __shared__ int64_t warp_excl[kWarps];
    __shared__ int64_t tile_excl;
    __shared__ unsigned long long tile_id;

    const int tid = threadIdx.x;
    const int w = tid >> 5;
    const unsigned lane = tid & 31;

    if (tid == 0) {
        tile_id = atomicAdd(a.ticket, 1ull);
        ki::mbar_init(&bar, 1);
        ki::fence_mbar_init();
    }
    __syncthreads();
    const uint64_t t = tile_id;
    const size_t first = (size_t)t * kTile;
    const int count = (int)min((size_t)kTile, a.n - first);
    const bool bulk = a.use_tma && count == kTile;

    if (bulk) {
        if (tid == 0) {
            ki::mbar_arrive_expect_tx(&bar, (uint32_t)kSmemBytes);
            ki::bulk_g2s(tile, a.in + first, (uint32_t)kSmemBytes, &bar);
        }
        if (!ki::mbar_wait_bounded(&bar, 0, a.status, a.timeout_ns)) {
            // The copy is still in flight: wait for it once more (bounded) before touching smem.
            ki::mbar_wait_bounded(&bar, 0, a.status, a.timeout_ns);
        }
    } else {
        for (int i = tid; i < kTile; i += kThreads) tile[i] = (i < count) ? a.in[first + i] : 0;
        __syncthreads();
    }

    // ---- pass 1: per-warp totals --------------------------------------------------------------
    const int64_t* wbase = tile + w * kWarpSpan;
    int64_t s = 0;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        const longlong2 v = *reinterpret_cast<const longlong2*>(wbase + 64 * j + 2 * lane);
        s = ki::wrap_add(s, ki::wrap_add(v.x, v.y));
    }
    s = ki::warpfold(s, ki::WrapAdd{});
    if (lane == 0) warp_tot[w] = s;
    __syncthreads();

    // ---- tile aggregate, lookback ---------------------------------------------------------------
    if (w == 0) {
        const int64_t v = (lane < (unsigned)kWarps) ? warp_tot[lane] : 0;
        const int64_t inc = ki::warpreduce(v, ki::WrapAdd{});
        if (lane < (unsigned)kWarps) warp_excl[lane] = ki::wrap_sub(inc, v);
        const int64_t agg = __shfl_sync(0xffffffffu, inc, kWarps - 1);
        const int64_t ex = ki::decoupled_lookback(a.st, t, agg, a.seed, a.status, a.timeout_ns);
        if (lane == 0) tile_excl = ex;
    }
    __syncthreads();

    // ---- pass 2: scan rows with @warpreduce -----------------------------------------------------
    int64_t carry = ki::wrap_add(tile_excl, warp_excl[w]);
    int64_t* wrow = tile + w * kWarpSpan;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        longlong2* p = reinterpret_cast<longlong2*>(wrow + 64 * j + 2 * lane);
        longlong2 v = *p;
        const int64_t pair = ki::wrap_add(v.x, v.y);
        const int64_t inc = ki::warpreduce(pair, ki::WrapAdd{});
        const int64_t o0 = ki::wrap_add(ki::wrap_add(carry, ki::wrap_sub(inc, pair)), v.x);
        v.y = ki::wrap_add(o0, v.y);
        v.x = o0;
        *p = v;
        carry = ki::wrap_add(carry, __shfl_sync(0xffffffffu, inc, 31));
    }

    if (bulk) {
        ki::fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            ki::bulk_s2g(a.out + first, tile, (uint32_t)kSmemBytes);
            ki::bulk_commit();
            ki::bulk_wait_all();
        }
    } else {
        __syncthreads();
        for (int i = tid; i < count; i += kThreads) a.out[first + i] = tile[i];
    }
}

}  // namespace

extern "C" int ki_scan_inclusive_i64(ki_ctx* ctx, const int64_t* d_in, int64_t* d_out, size_t n, int64_t seed,
                                     void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_in || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "scan: null pointer");
    if (!ki::aligned(d_in, 8) || !ki::aligned(d_out, 8))
        return ki::set_error(ctx, KI_ERR_ARG, "scan: Int64 pointers must be 8-byte aligned");
    if (d_in != d_out) {
        const uintptr_t i0 = (uintptr_t)d_in, o0 = (uintptr_t)d_out, nb = n * sizeof(int64_t);
        if (i0 < o0 + nb && o0 < i0 + nb)
            return ki::set_error(ctx, KI_ERR_ARG, "scan: partially overlapping input and output");
    }
    KI_GUARD(ctx);
    const size_t ntiles = (n + kTile - 1) / kTile;
    if (ntiles > (size_t)INT32_MAX) return ki::set_error(ctx, KI_ERR_ARG, "scan: n too large");
    // scratch: [ticket (256 B)] [flags ntiles] [aggs ntiles] [incls ntiles]
    const size_t flags_off = 256;
    const size_t bytes = flags_off + ntiles * 24;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_SCAN, bytes, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    cudaStream_t s = ki::as_stream(stream);
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, flags_off + ntiles * sizeof(uint64_t), s));

    KI_CUDA(ctx, cudaFuncSetAttribute(scan_i64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSmemBytes));
    ScanArgs a;
    a.in = d_in;
    a.out = d_out;
    a.n = n;
    a.seed = seed;
    a.st.flags = reinterpret_cast<uint64_t*>(b + flags_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + flags_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + flags_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.use_tma = ki::aligned(d_in, 16) && ki::aligned(d_out, 16);
    scan_i64_kernel<<<(unsigned)ntiles, kThreads, kSmemBytes, s>>>(a);
    return ki::check_launch(ctx, "scan_i64_kernel launch");
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc: code that runs while a CUDA graph is being captured, hosts
// whose memory is owned by another allocator (a Julia or Python pool that must not be bypassed), or
// real-time loops that forbid allocation after start-up.  ki_scan_inclusive_i64_noalloc runs the
// same kernel as ki_scan_inclusive_i64 but takes its tile-status scratch from the file-scope array
// below instead of a context, so it needs no context and allocates nothing.
//
// The array is sized for KI_SCAN_NOALLOC_MAX_N elements (65,536 tiles: a 256-byte header plus three
// 8-byte words per tile, about 1.5 MiB).  Every GPU that loads this library holds it until the
// process exits.  In host code the array's name is only a host-side stand-in, so its device address
// is looked up once per device with cudaGetSymbolAddress (with that device current) and cached; the
// first call on each device does this set-up and must therefore come before any stream capture.
// All calls share the array and it keeps the last call's contents: each call clears the ticket, the
// status word and the tile flags (cudaMemsetAsync on the cached address) before its launch, and
// calls that overlap on the GPU (different streams, or several host threads) race on it.
// A bounded wait that runs out is latched in the array's status word and not reported; use the
// context API where timeout reporting is needed.
// ---------------------------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocTiles = (KI_SCAN_NOALLOC_MAX_N + kTile - 1) / kTile;
constexpr size_t kNoAllocHeader = 256;  // ticket at 0, status word at 64
static __device__ __align__(256) unsigned char g_scan_noalloc_scratch[kNoAllocHeader + kNoAllocTiles * 24];

struct NoAllocDevice {
    bool ready = false;
    unsigned char* scratch = nullptr;
};
std::mutex g_noalloc_mutex;
NoAllocDevice g_noalloc_dev[64];

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
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KI_ERR_CUDA;
    unsigned char* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        NoAllocDevice& d = g_noalloc_dev[dev];
        if (!d.ready) {
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_scan_noalloc_scratch) != cudaSuccess || !p) return KI_ERR_CUDA;
            if (cudaFuncSetAttribute(scan_i64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSmemBytes) != cudaSuccess)
                return KI_ERR_CUDA;
            d.scratch = static_cast<unsigned char*>(p);
            d.ready = true;
        }
        scratch = d.scratch;
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
    a.st.flags = reinterpret_cast<uint64_t*>(scratch + kNoAllocHeader);
    a.st.aggs = reinterpret_cast<int64_t*>(scratch + kNoAllocHeader + kNoAllocTiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(scratch + kNoAllocHeader + kNoAllocTiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(scratch);
    a.status = reinterpret_cast<uint32_t*>(scratch + 64);
    a.timeout_ns = 2000000000ull;
    a.use_tma = ki::aligned(d_in, 16) && ki::aligned(d_out, 16);
    scan_i64_kernel<<<(unsigned)ntiles, kThreads, kSmemBytes, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? KI_OK : KI_ERR_CUDA;
}
