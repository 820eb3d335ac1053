// compact.cu -- order-preserving stream compaction: filter(x -> x > t, x) and findall.
//
// Persistent CTAs (3 per SM), software-pipelined over tiles of 16384 elements, with 8 "work" warps
// and one "look" warp, the same pipeline as scan.cu.  Iteration k of a CTA runs two phases:
//   phase A  work warps: wait for tile k (one 64 KiB 1-D TMA bulk copy, cp.async.bulk ...
//            mbarrier::complete_tx) and count its kept elements (warp w owns 2048 elements as 16 rows
//            of 32 lanes x float4: conflict-free 16-byte shared loads); warp 0 scans the 8 warp
//            counts with @warpreduce and publishes the tile count at once (ki/lookback.cuh);
//            look warp, at the same time: an L2 bulk prefetch of tile k-1 (cp.async.bulk.prefetch)
//            and the decoupled lookback of tile k-1;
//   phase B  the look warp takes the next ticket and starts its TMA into the free buffer;
//            work warps write tile k-1: re-read it from global memory (L2) and, for each row and
//            component c, take a @vote Ballot (ext/CUDA/shuffle_vote.jl:23-34, vote.sync ballot ->
//            UInt32).  An element's rank inside its row is
//                sum over c of popc(ballot_c & lanes_below) + (kept components before it in its lane)
//            which keeps source order (lane-major, then component).  The row's kept values and
//            indices go to a per-warp shared-memory run at their ranks (an element that is not kept
//            goes to its lane's discard slot, so there are no branches) and leave as coalesced
//            evict-first stores at tile prefix + warp prefix + row prefix.
// Between taking a ticket and publishing that tile's count a CTA only waits for its own load and
// its own second pass, never for a lookback.  Tiles that are partial or not 16-byte aligned are read
// with plain loads (padded with -Inf, which is never kept).
//
// Measured at n = 2^28 (0.467 ms, 0.57 of the copy peak): without the stores the same kernel takes
// 0.235 ms.  Writing the output streams evicts tiles that wait for their prefix, so most second-pass
// reads come back from DRAM; the prefetch turns them into one asynchronous bulk read per tile
// (0.51 -> 0.47 ms).  Slower alternatives: an evict-last or evict-first hint on the first read, tiles
// kept in shared memory (two or three buffers, fewer CTAs per SM), 4096/8192-element tiles, one or
// two CTAs per SM with more warps, looking tile k up right after its count, early tickets.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"

namespace {

#ifndef KI_COMPACT_LOOKBACK_K
#define KI_COMPACT_LOOKBACK_K 1
#endif
#ifndef KI_COMPACT_TILE
#define KI_COMPACT_TILE 16384
#endif
#ifndef KI_COMPACT_CTAS_PER_SM
#define KI_COMPACT_CTAS_PER_SM 3
#endif
#ifndef KI_COMPACT_WORK_WARPS
#define KI_COMPACT_WORK_WARPS 8
#endif
constexpr int kWorkWarps = KI_COMPACT_WORK_WARPS;
constexpr int kLookWarp = kWorkWarps;
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = kWorkThreads + 32;
constexpr int kTile = KI_COMPACT_TILE;
constexpr int kWarpSpan = kTile / kWorkWarps;   // elements per work warp
constexpr int kRows = kWarpSpan / 128;          // rows of 32 lanes x float4
static_assert(kWarpSpan % 128 == 0 && kWorkWarps <= 32, "tile must split into rows of 128 elements per warp");
constexpr int kBatch = kRows < 8 ? kRows : 8;   // rows loaded at once in the second pass
static_assert(kRows % kBatch == 0, "rows must split into whole batches");
// per warp: 128 values + 32 discard slots, then 128 indices + 32 discard slots
constexpr int kStageSlots = 160;
constexpr size_t kStageBytes = (size_t)kWorkWarps * kStageSlots * 8;
constexpr size_t kTileBytes = (size_t)kTile * sizeof(float);
constexpr size_t kSmemBytes = kTileBytes + kStageBytes;
constexpr int kLookbackK = KI_COMPACT_LOOKBACK_K;  // lookback window of 32*K tiles per round trip
constexpr int kCtasPerSm = KI_COMPACT_CTAS_PER_SM;

struct CompactArgs {
    const float* x;
    size_t n;
    float thr;
    float* out_vals;
    int32_t* out_idx;
    int64_t index_base;
    uint64_t* d_count;
    ki::TileStatus st;
    unsigned long long* ticket;
    uint32_t* status;
    uint64_t timeout_ns;
    int tma_in;  // x is 16-byte aligned: full tiles come in by TMA, rows by float4
};

struct Pending {
    unsigned long long t;
    int64_t agg;
    int64_t tile_excl;
    int warp_excl[kWorkWarps];
};

__device__ __forceinline__ void work_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkThreads) : "memory"); }

__device__ __forceinline__ int kept4(const float4& v, float thr) {
    return (v.x > thr) + (v.y > thr) + (v.z > thr) + (v.w > thr);
}

// VALS / IDX: which outputs are written (an absent output costs no instructions).
template <bool VALS, bool IDX>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) compact_gt_f32_kernel(CompactArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float* sb = reinterpret_cast<float*>(smem_raw);
    __shared__ __align__(8) uint64_t bar;
    __shared__ int warp_cnt[kWorkWarps];
    __shared__ Pending slot[2];  // tile k (being counted) and tile k-1 (being written)
    __shared__ unsigned long long ticket;

    const int tid = threadIdx.x;
    const int w = tid >> 5;
    const unsigned lane = tid & 31;
    const uint64_t ntiles = (a.n + kTile - 1) / kTile;
    auto bulk_ok = [&](uint64_t t) { return a.tma_in && t < ntiles && (t + 1) * (uint64_t)kTile <= a.n; };
    auto fetch = [&]() {  // take a ticket and start its load (one thread)
        const unsigned long long t = atomicAdd(a.ticket, 1ull);
        ticket = t;
        if (bulk_ok(t)) {
            ki::fence_proxy_async_smem();  // earlier generic reads of sb come first
            ki::mbar_arrive_expect_tx(&bar, (uint32_t)kTileBytes);
            ki::bulk_g2s(sb, a.x + t * kTile, (uint32_t)kTileBytes, &bar);
        }
    };
    if (tid == 0) {
        ki::mbar_init(&bar, 1);
        ki::fence_mbar_init();
        fetch();
    }
    __syncthreads();

    const unsigned below = (1u << lane) - 1u;  // lanes with a lower index
    const float thr = a.thr;
    uint32_t phase = 0;
    bool have_old = false;
    int cur = 0;  // slot of tile k; tile k-1 is in slot cur ^ 1
    while (true) {
        const uint64_t t_new = ticket;
        const bool new_valid = t_new < ntiles;
        if (!new_valid && !have_old) break;

        // ---- phase A: count and publish tile k  ||  prefetch and look back for tile k-1 ------------
        if (w == kLookWarp) {
            if (have_old) {
                Pending& o = slot[cur ^ 1];
                // bring tile k-1 back into L2 (if it left) while its prefix is looked up
                if (lane == 0 && bulk_ok(o.t)) ki::bulk_prefetch_l2(a.x + o.t * kTile, (uint32_t)kTileBytes);
                const int64_t ex = ki::decoupled_lookback<kLookbackK>(a.st, o.t, o.agg, 0, a.status, a.timeout_ns);
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
                // partial or unaligned tile: plain loads, padded with values that are never kept
                for (int i = tid; i < kTile; i += kWorkThreads) sb[i] = (i < count) ? a.x[first + i] : -INFINITY;
                work_sync();
            }
            const float4* row0 = reinterpret_cast<const float4*>(sb + w * kWarpSpan) + lane;
            int c = 0;
#pragma unroll 8
            for (int j = 0; j < kRows; ++j) c += kept4(row0[32 * j], thr);
            c = ki::warpfold(c, ki::Add{});
            if (lane == 0) warp_cnt[w] = c;
            work_sync();
            if (w == 0) {
                const int x = (lane < (unsigned)kWorkWarps) ? warp_cnt[lane] : 0;
                const int inc = ki::warpreduce(x, ki::Add{});
                const int agg = __shfl_sync(0xffffffffu, inc, kWorkWarps - 1);
                Pending& e = slot[cur];
                if (lane < (unsigned)kWorkWarps) e.warp_excl[lane] = inc - x;
                if (lane == 0) {
                    e.t = t_new;
                    e.agg = agg;
                    ki::publish_aggregate(a.st, t_new, agg, 0);
                }
            }
        }
        __syncthreads();  // tile k counted (buffer free, slot written); tile k-1's prefix known

        // ---- phase B: start tile k+1's load; write tile k-1 -------------------------------------------
        if (tid == kLookWarp * 32 && new_valid) fetch();  // the look warp is idle in phase B
        if (w < kWorkWarps && have_old) {
            const Pending& o = slot[cur ^ 1];
            const size_t first = (size_t)o.t * kTile;
            const int count = (int)min((size_t)kTile, a.n - first);
            const bool vec_in = a.tma_in && count == kTile;
            // outputs of this warp start at one pointer; offsets from it fit 32 bits
            const int64_t at = o.tile_excl + o.warp_excl[w];
            float* vals = VALS ? a.out_vals + at : nullptr;
            int32_t* idxs = IDX ? a.out_idx + at : nullptr;
            const int i_lane = w * kWarpSpan + 4 * (int)lane;  // element of (row 0, component 0)
            // output index of that element; unsigned, so the padding past the last element wraps
            // harmlessly instead of overflowing (it is never stored)
            const uint32_t ix0 = (uint32_t)((int64_t)first + a.index_base) + (uint32_t)i_lane;
            float* sv = reinterpret_cast<float*>(smem_raw + kTileBytes) + w * 2 * kStageSlots;
            int32_t* si = reinterpret_cast<int32_t*>(sv + kStageSlots);
            int pos = 0;
#pragma unroll 1
            for (int j0 = 0; j0 < kRows; j0 += kBatch) {
                float4 v[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {  // a batch of loads in flight first
                    const int i0 = i_lane + 128 * (j0 + j);
                    if (vec_in) {
                        v[j] = *reinterpret_cast<const float4*>(a.x + first + i0);
                    } else {
                        v[j].x = (i0 + 0 < count) ? a.x[first + i0 + 0] : -INFINITY;
                        v[j].y = (i0 + 1 < count) ? a.x[first + i0 + 1] : -INFINITY;
                        v[j].z = (i0 + 2 < count) ? a.x[first + i0 + 2] : -INFINITY;
                        v[j].w = (i0 + 3 < count) ? a.x[first + i0 + 3] : -INFINITY;
                    }
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const bool p0 = v[j].x > thr, p1 = v[j].y > thr, p2 = v[j].z > thr, p3 = v[j].w > thr;
                    const unsigned b0 = ki::ballot(p0), b1 = ki::ballot(p1), b2 = ki::ballot(p2), b3 = ki::ballot(p3);
                    const int ahead = __popc(b0 & below) + __popc(b1 & below) + __popc(b2 & below) + __popc(b3 & below);
                    const int row = __popc(b0) + __popc(b1) + __popc(b2) + __popc(b3);
                    const uint32_t ix = ix0 + 128u * (uint32_t)(j0 + j);
                    // the row's kept elements, in source order, as one run in this warp's stage ...
                    const int r0 = ahead, r1 = r0 + (int)p0, r2 = r1 + (int)p1, r3 = r2 + (int)p2;
                    const int junk = 128 + (int)lane;
                    if (VALS) {
                        sv[p0 ? r0 : junk] = v[j].x;
                        sv[p1 ? r1 : junk] = v[j].y;
                        sv[p2 ? r2 : junk] = v[j].z;
                        sv[p3 ? r3 : junk] = v[j].w;
                    }
                    if (IDX) {
                        si[p0 ? r0 : junk] = (int32_t)ix;
                        si[p1 ? r1 : junk] = (int32_t)(ix + 1u);
                        si[p2 ? r2 : junk] = (int32_t)(ix + 2u);
                        si[p3 ? r3 : junk] = (int32_t)(ix + 3u);
                    }
                    __syncwarp();
                    // ... written out with consecutive lanes on consecutive addresses
                    for (int e = (int)lane; e < row; e += 32) {
                        if (VALS) __stcs(vals + pos + e, sv[e]);
                        if (IDX) __stcs(idxs + pos + e, si[e]);
                    }
                    __syncwarp();
                    pos += row;
                }
            }
            if (o.t == ntiles - 1 && w == 0 && lane == 0 && a.d_count) *a.d_count = (uint64_t)(o.tile_excl + o.agg);
        }
        __syncthreads();  // the next ticket is visible; slot cur ^ 1 is free
        have_old = new_valid;
        cur ^= 1;
    }
}

template <bool VALS, bool IDX>
int launch_compact(ki_ctx* ctx, const CompactArgs& a, size_t grid, cudaStream_t s) {
    KI_CUDA(ctx, cudaFuncSetAttribute(compact_gt_f32_kernel<VALS, IDX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSmemBytes));
    compact_gt_f32_kernel<VALS, IDX><<<(unsigned)grid, kThreads, kSmemBytes, s>>>(a);
    return ki::check_launch(ctx, "compact_gt_f32_kernel launch");
}

}  // namespace

extern "C" int ki_compact_gt_f32(ki_ctx* ctx, const float* d_x, size_t n, float threshold, float* d_out_vals,
                                 int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "compact: null input");
    if (n > 0 && !ki::aligned(d_x, 4)) return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned Float32 input");
    if ((d_out_vals && !ki::aligned(d_out_vals, 4)) || (d_out_idx && !ki::aligned(d_out_idx, 4)))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned output");
    if (index_base < INT32_MIN || (n > 0 && index_base + (int64_t)n - 1 > (int64_t)INT32_MAX))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: indices do not fit Int32");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    if (n == 0) {
        if (d_count) KI_CUDA(ctx, cudaMemsetAsync(d_count, 0, sizeof(uint64_t), s));
        return KI_OK;
    }
    const size_t ntiles = (n + kTile - 1) / kTile;
    const size_t words_off = 256;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_COMPACT, words_off + ntiles * 24, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, words_off + ntiles * sizeof(uint64_t), s));
    CompactArgs a;
    a.x = d_x;
    a.n = n;
    a.thr = threshold;
    a.out_vals = d_out_vals;
    a.out_idx = d_out_idx;
    a.index_base = index_base;
    a.d_count = d_count;
    a.st.words = reinterpret_cast<uint64_t*>(b + words_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + words_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + words_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.tma_in = ki::aligned(d_x, 16);
    size_t grid = (size_t)ctx->sm_count * kCtasPerSm;
    if (grid > ntiles) grid = ntiles;
    if (d_out_vals && d_out_idx) return launch_compact<true, true>(ctx, a, grid, s);
    if (d_out_vals) return launch_compact<true, false>(ctx, a, grid, s);
    if (d_out_idx) return launch_compact<false, true>(ctx, a, grid, s);
    return launch_compact<false, false>(ctx, a, grid, s);
}
