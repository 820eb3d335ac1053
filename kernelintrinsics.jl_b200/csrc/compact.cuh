// compact.cuh -- order-preserving stream compaction: filter(v -> v op t, x) and findall(v -> v op t, x)
// for op in >, >=, <, <=, ==, != over Int32, UInt32, Int64, UInt64, Float32 and Float64 (IEEE
// comparisons, as Base's operators).
//
// Persistent CTAs (3 per SM), software-pipelined over 64 KiB tiles (16384 4-byte or 8192 8-byte
// elements; the description below counts 4-byte elements), with 8 "work" warps
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
//            indices go to a per-warp shared-memory stage at their ranks, where slot s holds output
//            element G + s with G a multiple of 32: every run of 32 that fills up leaves as one whole,
//            aligned line per output (evict-first stores) and the rest moves to the front of the stage.
// Between taking a ticket and publishing that tile's count a CTA only waits for its own load and
// its own second pass, never for a lookback.  Tiles that are not 16-byte aligned are read with plain
// loads; in the partial last tile, elements past the end are excluded explicitly.
//
// Measured at n = 2^28: 0.427 ms (0.62 of the copy peak), with Float32 / 4-byte values staged as
// one 8-byte {value, index} slot per element, the row's count taken from lane 31's rank by one
// shuffle (not four popc) and second-pass batches of 4 rows (0.435 ms with two 4-byte stage arrays,
// four popc and batches of 8; packed slots with batches of 8 spill: 0.443).  Writing each row's run
// out on its own (unaligned 4-byte stores, most lines written in two parts by two store
// instructions) took 0.471 ms; with whole aligned lines (and the two stage arrays), plain stores in
// place of evict-first ones 0.443, an evict-last tile load with evict-first second reads 0.474, no
// L2 prefetch 0.510, two CTAs of 16 warps over 8-row
// spans 0.437, batches of 4 rows 0.437, lookback windows of 64 / 128 tiles 0.439 / 0.454, runs
// written by bulk copies from the stage (each row then waits for its copy to read the stage) 0.70.
// Without the barrier at the end of each iteration (the next ticket delivered through the tile
// mbarrier, three pending-tile slots) 0.518 ms, and 0.438 with two CTAs of 16 warps.
// Taking each ticket one fetch early and bulk-prefetching its tile into L2 (so that the tile's
// load later hits L2): 0.549 ms; a tile then waits longer for its count, and so do the lookbacks
// of the tiles after it.
// A lookback window that doubles (32, 64, 128 tiles per round trip) while it finds no inclusive
// prefix: 0.428-0.434 ms at 2^28 and 78 us against 76 at 2^25; the waits are for predecessors
// that have not published yet, not for long walks back.
// Second-pass reads hit L2 only while at most about 96 KiB of tiles per SM are in flight (48 KiB
// tiles x 2 CTAs of 16 warps, 32 KiB x 3 CTAs, 36 KiB x 3 CTAs of 12 warps), and each of those
// shapes is slower (0.47-0.51 ms): fewer bytes or warps in flight cost more than the re-reads.
// The lookback's waits cost about 5 % (0.414 ms with a made-up prefix and no lookback).  The
// figures below were taken with the per-row write-out:
// without the stores the kernel takes 0.235 ms.  Writing the output streams evicts tiles that wait
// for their prefix, so most second-pass reads come back from DRAM; the prefetch turns them into one
// asynchronous bulk read per tile (0.51 -> 0.47 ms).  Slower alternatives: an evict-last or
// evict-first hint on the first read (also with the lines demoted to normal priority after the
// second read: 0.48 ms), evict-first second
// reads (0.50), tiles kept in shared memory (two or three buffers, fewer CTAs per SM), 4096/8192-
// element tiles, one CTA per SM of 16 or 24 work warps over 128/192 KiB tiles (0.52-0.54), two CTAs
// per SM of 16 warps over 64 KiB tiles (0.47-0.48), 16 rows in flight per warp in the second pass
// (0.54: spills), two CTAs of 12 warps over 48 KiB tiles (0.51), looking tile k up right after its
// count, early tickets, and compacting each tile into shared memory right after its count so that
// its write-out reads no global memory (32 KiB tiles double-buffered, a tile-sized compacted buffer
// with 16-bit indices, 2 CTAs per SM: 0.645 ms; the extra pass and the smaller tiles in flight cost
// more than the re-reads).  L2 eviction-priority policies do not change it either (2^28, median of
// 20): evict_normal on the tile load 0.468 ms (0.469 without), evict_first on it 0.480, evict_first
// policy on the output stores 0.485, plain stores 0.474, evict_first policy on the second-pass loads
// as well 0.52, no L2 prefetch 0.535; the Int64 scan's hints (evict-last tile load, streaming
// re-read) 0.51, and with its shape (one CTA of 31 work warps, 124 KiB tiles) 0.49.  Tiles kept in
// shared memory with each warp refilling its span of the buffer as soon as it is written (two 32 KiB
// buffers, 3 CTAs per SM) 0.59 ms; 64 KiB x 1 CTA 0.92; 16 KiB x 4 CTAs 0.73; 48 KiB x 2 CTAs 0.63.
// Tiles held in registers (one CTA of 31 work warps per SM, each thread keeping its 16 values of
// tile k and of tile k-1, a 3-stage TMA ring of 62 KiB tiles, the lookbacks run by a look warp
// decoupled through mbarriers): 0.61-0.63 ms, and 1.04 ms with 31 KiB tiles: without a second pass
// the DRAM bytes are the algorithmic ones, but each CTA then waits for its tile's prefix, and the
// lookback chain over the ~150 tiles in flight sets the pace.  Every variant was checked against
// this kernel's output (small, partial, misaligned and 2^28 inputs) before timing.  The kernel is
// latency-bound (ncu at 2^26: DRAM 65 %, issue 50 %, warps 41 % active, stalls mostly at
// barriers).  KI_COMPACT_WORK_WARPS, KI_COMPACT_ROWS and KI_COMPACT_CTAS_PER_SM set the shape.
#pragma once

#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"
#include "ki/ops.cuh"

namespace {

#ifndef KI_COMPACT_LOOKBACK_K
#define KI_COMPACT_LOOKBACK_K 1
#endif
#ifndef KI_COMPACT_PREFETCH
#define KI_COMPACT_PREFETCH 1
#endif
#ifndef KI_COMPACT_CTAS_PER_SM
#define KI_COMPACT_CTAS_PER_SM 3
#endif
#ifndef KI_COMPACT_WORK_WARPS
#define KI_COMPACT_WORK_WARPS 8
#endif
#ifndef KI_COMPACT_ROWS
#define KI_COMPACT_ROWS 16
#endif
constexpr int kWorkWarps = KI_COMPACT_WORK_WARPS;
constexpr int kLookWarp = kWorkWarps;
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = kWorkThreads + 32;
constexpr int kRows = KI_COMPACT_ROWS;  // rows of 32 lanes x one 16-byte vector per work warp
constexpr size_t kTileBytes = (size_t)kWorkWarps * kRows * 512;  // 64 KiB: 16384 elements of 4 bytes or 8192 of 8
#ifndef KI_COMPACT_BATCH
#define KI_COMPACT_BATCH 4
#endif
constexpr int kBatch = KI_COMPACT_BATCH;  // rows loaded at once in the second pass
static_assert(kRows % kBatch == 0, "the second pass loads whole batches of rows");
constexpr int kLookbackK = KI_COMPACT_LOOKBACK_K;  // lookback window of 32*K tiles per round trip
constexpr int kCtasPerSm = KI_COMPACT_CTAS_PER_SM;

template <class T>
struct CShape {
    static constexpr int kE = (int)(16 / sizeof(T));         // elements per lane per row
    static constexpr int kRow = 32 * kE;                      // elements per row
    static constexpr int kSpan = kRows * kRow;                 // elements per work warp
    static constexpr int kTile = kWorkWarps * kSpan;           // elements per tile
    static constexpr int kStageSlots = kRow + 32;              // up to 31 carried over + one row's run
    static constexpr size_t kStageBytes = (size_t)kWorkWarps * kStageSlots * (sizeof(T) + sizeof(int32_t));
    static constexpr size_t kSmemBytes = kTileBytes + kStageBytes;
    static_assert(kTile * sizeof(T) == kTileBytes, "tile layout");
};

// Comparison predicates (x op t), IEEE semantics for floats as Base's <, <=, ==, != and >.
struct PGt { template <class T> __device__ static __forceinline__ bool test(T x, T t) { return x > t; } };
struct PGe { template <class T> __device__ static __forceinline__ bool test(T x, T t) { return x >= t; } };
struct PLt { template <class T> __device__ static __forceinline__ bool test(T x, T t) { return x < t; } };
struct PLe { template <class T> __device__ static __forceinline__ bool test(T x, T t) { return x <= t; } };
struct PEq { template <class T> __device__ static __forceinline__ bool test(T x, T t) { return x == t; } };
struct PNe { template <class T> __device__ static __forceinline__ bool test(T x, T t) { return x != t; } };

template <class T>
__device__ __forceinline__ uint32_t bits32(T v) {
    static_assert(sizeof(T) == 4, "4-byte values");
    uint32_t u;
    memcpy(&u, &v, 4);
    return u;
}

struct CompactArgs {
    const void* x;
    size_t n;
    uint64_t thr_bits;  // the threshold, as a T
    void* out_vals;
    int32_t* out_idx;
    int64_t index_base;
    uint64_t* d_count;
    ki::TileStatus st;
    unsigned long long* ticket;
    uint32_t* status;
    uint64_t timeout_ns;
    int tma_in;  // x is 16-byte aligned: full tiles come in by TMA, rows as 16-byte vectors
};

struct Pending {
    unsigned long long t;
    int64_t agg;
    int64_t tile_excl;
    int warp_excl[kWorkWarps];
};

__device__ __forceinline__ void work_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkThreads) : "memory"); }

// T: element type; P: predicate; VALS / IDX: which outputs are written (an absent output costs no
// instructions).
template <class T, class P, bool VALS, bool IDX>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) compact_kernel(CompactArgs a) {
    using S = CShape<T>;
    using V = ki::Vec16<T>;
    constexpr int kE = S::kE;
    constexpr int kTile = S::kTile;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    T* sb = reinterpret_cast<T*>(smem_raw);
    __shared__ __align__(8) uint64_t bar;
    __shared__ int warp_cnt[kWorkWarps];
    __shared__ Pending slot[2];  // tile k (being counted) and tile k-1 (being written)
    __shared__ unsigned long long ticket;

    const T* x = static_cast<const T*>(a.x);
    const T thr = ki::from_bits<T>(a.thr_bits);
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
            ki::bulk_g2s(sb, x + t * kTile, (uint32_t)kTileBytes, &bar);
        }
    };
    if (tid == 0) {
        ki::mbar_init(&bar, 1);
        ki::fence_mbar_init();
        fetch();
    }
    __syncthreads();

    const unsigned below = (1u << lane) - 1u;  // lanes with a lower index
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
                if (KI_COMPACT_PREFETCH && lane == 0 && bulk_ok(o.t))
                    ki::bulk_prefetch_l2(x + o.t * kTile, (uint32_t)kTileBytes);
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
                for (int i = tid; i < kTile; i += kWorkThreads) sb[i] = (i < count) ? x[first + i] : T(0);
                work_sync();
            }
            const V* row0 = reinterpret_cast<const V*>(sb + w * S::kSpan) + lane;
            int c = 0;
            if (count == kTile) {
#pragma unroll 8
                for (int j = 0; j < kRows; ++j) {
                    const V v = row0[32 * j];
#pragma unroll
                    for (int e = 0; e < kE; ++e) c += P::test(v.v[e], thr);
                }
            } else {  // the partial last tile: elements past count do not exist
                const int i_lane = w * S::kSpan + kE * (int)lane;
                for (int j = 0; j < kRows; ++j) {
                    const V v = row0[32 * j];
#pragma unroll
                    for (int e = 0; e < kE; ++e) c += (i_lane + S::kRow * j + e < count) && P::test(v.v[e], thr);
                }
            }
            c = ki::warpfold(c, ki::Add{});
            if (lane == 0) warp_cnt[w] = c;
            work_sync();
            if (w == 0) {
                const int xx = (lane < (unsigned)kWorkWarps) ? warp_cnt[lane] : 0;
                const int inc = ki::warpreduce(xx, ki::Add{});
                const int agg = __shfl_sync(0xffffffffu, inc, kWorkWarps - 1);
                Pending& e = slot[cur];
                if (lane < (unsigned)kWorkWarps) e.warp_excl[lane] = inc - xx;
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
            const bool full = count == kTile;
            const bool vec_in = a.tma_in;
            // this warp's outputs start at element `at`; the stage is aligned to 32 elements below it
            const int64_t at = o.tile_excl + o.warp_excl[w];
            const int i_lane = w * S::kSpan + kE * (int)lane;  // element of (row 0, component 0)
            // output index of that element; unsigned, so indices past the last element wrap
            // harmlessly instead of overflowing (they are never stored)
            const uint32_t ix0 = (uint32_t)((int64_t)first + a.index_base) + (uint32_t)i_lane;
            T* sv = reinterpret_cast<T*>(smem_raw + kTileBytes) + (size_t)w * S::kStageSlots;
            int32_t* si = reinterpret_cast<int32_t*>(smem_raw + kTileBytes + (size_t)kWorkWarps * S::kStageSlots * sizeof(T)) +
                          (size_t)w * S::kStageSlots;
            // 4-byte elements with both outputs: one 8-byte {value bits, index} slot per element (one
            // shared store and load per element instead of two)
            constexpr bool kPack = sizeof(T) == 4 && VALS && IDX;
            uint2* sp = reinterpret_cast<uint2*>(smem_raw + kTileBytes) + (size_t)w * S::kStageSlots;
            // slot s of the stage holds output element G + s (G a multiple of 32); slots below `lo` belong
            // to the previous warp's run and are never stored
            int L = (int)(at & 31);  // slots in use
            int lo = L;
            T* vbase = VALS ? static_cast<T*>(a.out_vals) + (at - L) : nullptr;
            int32_t* ibase = IDX ? a.out_idx + (at - L) : nullptr;
            // FULL: a whole tile (no element past the end), the common case, without bounds checks
            auto rows_pass = [&](auto full_tag) {
                constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll 1
                for (int j0 = 0; j0 < kRows; j0 += kBatch) {
                    V v[kBatch];
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {  // a batch of loads in flight first
                        const int i0 = i_lane + S::kRow * (j0 + j);
                        if (FULL && vec_in) {
                            const uint4 raw = *reinterpret_cast<const uint4*>(x + first + i0);
                            v[j] = *reinterpret_cast<const V*>(&raw);
                        } else {
#pragma unroll
                            for (int e = 0; e < kE; ++e) v[j].v[e] = (FULL || i0 + e < count) ? x[first + i0 + e] : T(0);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        const int i0 = i_lane + S::kRow * (j0 + j);
                        bool p[kE];
                        unsigned b[kE];
                        int ahead = 0;
#pragma unroll
                        for (int e = 0; e < kE; ++e) {
                            p[e] = P::test(v[j].v[e], thr);
                            if (!FULL) p[e] = p[e] && (i0 + e < count);
                            b[e] = ki::ballot(p[e]);
                            ahead += __popc(b[e] & below);
                        }
                        const uint32_t ix = ix0 + (uint32_t)(S::kRow * (j0 + j));
                        // the row's kept elements, in source order, after the ones carried over
                        int r = L + ahead;
#pragma unroll
                        for (int e = 0; e < kE; ++e) {
                            if (p[e]) {
                                if constexpr (kPack) {
                                    sp[r] = make_uint2(bits32(v[j].v[e]), ix + (uint32_t)e);
                                } else {
                                    if (VALS) sv[r] = v[j].v[e];
                                    if (IDX) si[r] = (int32_t)(ix + (uint32_t)e);
                                }
                            }
                            r += (int)p[e];
                        }
                        const int row = __shfl_sync(0xffffffffu, r, 31) - L;  // kept in this row
                        __syncwarp();
                        const int total = L + row;
                        const int full_runs = total >> 5;
                        if (full_runs > 0) {
                            // whole runs of 32 leave as aligned lines, consecutive lanes on consecutive addresses
                            for (int c = 0; c < full_runs; ++c) {
                                const int sl = 32 * c + (int)lane;
                                if (sl >= lo) {
                                    if constexpr (kPack) {
                                        const uint2 q = sp[sl];
                                        __stcs(vbase + sl, ki::from_bits<T>(q.x));
                                        __stcs(ibase + sl, (int32_t)q.y);
                                    } else {
                                        if (VALS) __stcs(vbase + sl, sv[sl]);
                                        if (IDX) __stcs(ibase + sl, si[sl]);
                                    }
                                }
                            }
                            // the remainder (< 32) moves to the front
                            const int rem = total - 32 * full_runs;
                            if constexpr (kPack) {
                                uint2 tq = make_uint2(0u, 0u);
                                if ((int)lane < rem) tq = sp[32 * full_runs + lane];
                                __syncwarp();
                                if ((int)lane < rem) sp[lane] = tq;
                            } else {
                                T tv{};
                                int32_t ti = 0;
                                if ((int)lane < rem) {
                                    if (VALS) tv = sv[32 * full_runs + lane];
                                    if (IDX) ti = si[32 * full_runs + lane];
                                }
                                __syncwarp();
                                if ((int)lane < rem) {
                                    if (VALS) sv[lane] = tv;
                                    if (IDX) si[lane] = ti;
                                }
                            }
                            if (VALS) vbase += 32 * full_runs;
                            if (IDX) ibase += 32 * full_runs;
                            lo = 0;
                            L = rem;
                            __syncwarp();
                        } else {
                            L = total;
                        }
                    }
                }
            };
            if (full) rows_pass(std::true_type{});
            else rows_pass(std::false_type{});
            if ((int)lane >= lo && (int)lane < L) {  // the last, partial run
                if constexpr (kPack) {
                    const uint2 q = sp[lane];
                    __stcs(vbase + lane, ki::from_bits<T>(q.x));
                    __stcs(ibase + lane, (int32_t)q.y);
                } else {
                    if (VALS) __stcs(vbase + lane, sv[lane]);
                    if (IDX) __stcs(ibase + lane, si[lane]);
                }
            }
            if (o.t == ntiles - 1 && w == 0 && lane == 0 && a.d_count) *a.d_count = (uint64_t)(o.tile_excl + o.agg);
        }
        __syncthreads();  // the next ticket is visible; slot cur ^ 1 is free
        have_old = new_valid;
        cur ^= 1;
    }
}

template <class T, class P, bool VALS, bool IDX>
int launch_compact(ki_ctx* ctx, const CompactArgs& a, size_t grid, cudaStream_t s) {
    constexpr size_t smem = CShape<T>::kSmemBytes;
    KI_CUDA(ctx, cudaFuncSetAttribute(compact_kernel<T, P, VALS, IDX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    compact_kernel<T, P, VALS, IDX><<<(unsigned)grid, kThreads, smem, s>>>(a);
    return ki::check_launch(ctx, "compact_kernel launch");
}

// count(v -> v op t, x): with neither output asked for, order does not matter, so no tiles and no
// lookback: every thread counts its 16-byte vectors (four in flight), warps add their counts with
// @warpfold and each block adds its total to the 64-bit result with one atomic (integer addition,
// so the result does not depend on the order).
constexpr int kCountThreads = 256;
constexpr int kCountUnroll = 4;

template <class T, class P>
__global__ void __launch_bounds__(kCountThreads) count_kernel(const T* __restrict__ x, size_t head, size_t nvec, size_t n,
                                                              uint64_t thr_bits, unsigned long long* count) {
    const T thr = ki::from_bits<T>(thr_bits);
    constexpr int kE = (int)(16 / sizeof(T));
    const uint4* xv = reinterpret_cast<const uint4*>(x + head);
    const size_t stride = (size_t)gridDim.x * kCountThreads;
    size_t i = (size_t)blockIdx.x * kCountThreads + threadIdx.x;
    unsigned c = 0;
    for (; i + (kCountUnroll - 1) * stride < nvec; i += kCountUnroll * stride) {
        ki::Packed16<T> v[kCountUnroll];
#pragma unroll
        for (int u = 0; u < kCountUnroll; ++u) v[u].raw = __ldcs(xv + i + u * stride);
#pragma unroll
        for (int u = 0; u < kCountUnroll; ++u)
#pragma unroll
            for (int e = 0; e < kE; ++e) c += P::test(v[u].get(e), thr);
    }
    for (; i < nvec; i += stride) {
        ki::Packed16<T> v;
        v.raw = __ldcs(xv + i);
#pragma unroll
        for (int e = 0; e < kE; ++e) c += P::test(v.get(e), thr);
    }
    if (blockIdx.x == 0) {  // unaligned head and the tail (each < one vector)
        const size_t tail0 = head + nvec * kE;
        const size_t t = threadIdx.x;
        if (t < head) c += P::test(x[t], thr);
        if (t < n - tail0) c += P::test(x[tail0 + t], thr);
    }
    __shared__ unsigned long long warp_sum[kCountThreads / 32];
    const unsigned long long wsum = ki::warpfold((unsigned long long)c, ki::Add{});
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = wsum;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (int w = 0; w < kCountThreads / 32; ++w) b += warp_sum[w];
        if (b) atomicAdd(count, b);
    }
}

template <class T, class P>
int count_run(ki_ctx* ctx, const T* x, size_t n, uint64_t thr_bits, uint64_t* d_count, cudaStream_t s) {
    KI_CUDA(ctx, cudaMemsetAsync(d_count, 0, sizeof(uint64_t), s));
    if (n == 0) return KI_OK;
    constexpr int kE = (int)(16 / sizeof(T));
    size_t head = (size_t)((16 - (reinterpret_cast<uintptr_t>(x) & 15)) & 15) / sizeof(T);
    if (head > n) head = n;
    const size_t nvec = (n - head) / kE;
    size_t blocks = (nvec + (size_t)kCountThreads * kCountUnroll - 1) / ((size_t)kCountThreads * kCountUnroll);
    const size_t cap = (size_t)ctx->sm_count * (2048 / kCountThreads);
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    count_kernel<T, P><<<(unsigned)blocks, kCountThreads, 0, s>>>(x, head, nvec, n, thr_bits,
                                                                  reinterpret_cast<unsigned long long*>(d_count));
    return ki::check_launch(ctx, "count_kernel launch");
}

template <class T, class P>
int compact_run(ki_ctx* ctx, const void* d_x, size_t n, const void* h_thr, void* d_out_vals, int32_t* d_out_idx,
                int64_t index_base, uint64_t* d_count, cudaStream_t s) {
    constexpr int kTile = CShape<T>::kTile;
    if (n > 0 && !ki::aligned(d_x, sizeof(T))) return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned input");
    if ((d_out_vals && !ki::aligned(d_out_vals, sizeof(T))) || (d_out_idx && !ki::aligned(d_out_idx, 4)))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: misaligned output");
    if (!d_out_vals && !d_out_idx) {  // a count
        if (!d_count) return KI_OK;
        uint64_t thr_bits = 0;
        memcpy(&thr_bits, h_thr, sizeof(T));
        return count_run<T, P>(ctx, static_cast<const T*>(d_x), n, thr_bits, d_count, s);
    }
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
    a.thr_bits = 0;
    memcpy(&a.thr_bits, h_thr, sizeof(T));
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
    if (d_out_vals && d_out_idx) return launch_compact<T, P, true, true>(ctx, a, grid, s);
    if (d_out_vals) return launch_compact<T, P, true, false>(ctx, a, grid, s);
    return launch_compact<T, P, false, true>(ctx, a, grid, s);  // (no output at all is a count)
}

// P tested on M(x): filter(v -> f(v) op t, x) keeps x itself, so the kernel writes the element, not
// its map.
template <class M, class P>
struct PMapped {
    template <class T>
    __device__ static __forceinline__ bool test(T x, T t) { return P::test(M::apply(x), t); }
};
template <class M, class P>
using PredOf = typename std::conditional<std::is_same<M, ki::MapId>::value, P, PMapped<M, P>>::type;

template <class T, class M = ki::MapId>
int compact_pred(ki_ctx* ctx, int pred, const void* d_x, size_t n, const void* h_thr, void* d_out_vals,
                 int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, cudaStream_t s) {
    switch (pred) {
        case KI_PRED_GT: return compact_run<T, PredOf<M, PGt>>(ctx, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_PRED_GE: return compact_run<T, PredOf<M, PGe>>(ctx, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_PRED_LT: return compact_run<T, PredOf<M, PLt>>(ctx, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_PRED_LE: return compact_run<T, PredOf<M, PLe>>(ctx, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_PRED_EQ: return compact_run<T, PredOf<M, PEq>>(ctx, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_PRED_NE: return compact_run<T, PredOf<M, PNe>>(ctx, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "compact: unknown predicate");
    }
}

template <class M = ki::MapId>
int compact_dtype(ki_ctx* ctx, int pred, int dtype, const void* d_x, size_t n, const void* h_thr, void* d_out_vals,
                  int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, cudaStream_t s) {
    switch (dtype) {
        case KI_I32: return compact_pred<int32_t, M>(ctx, pred, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_U32: return compact_pred<uint32_t, M>(ctx, pred, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_I64: return compact_pred<int64_t, M>(ctx, pred, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_U64: return compact_pred<uint64_t, M>(ctx, pred, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_F32: return compact_pred<float, M>(ctx, pred, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        case KI_F64: return compact_pred<double, M>(ctx, pred, d_x, n, h_thr, d_out_vals, d_out_idx, index_base, d_count, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "compact: dtype must be Int32/UInt32/Int64/UInt64/Float32/Float64");
    }
}

inline int check_common(ki_ctx* ctx, const void* d_x, size_t n, int64_t index_base) {
    if (n > 0 && !d_x) return ki::set_error(ctx, KI_ERR_ARG, "compact: null input");
    if (index_base < INT32_MIN || (n > 0 && index_base + (int64_t)n - 1 > (int64_t)INT32_MAX))
        return ki::set_error(ctx, KI_ERR_ARG, "compact: indices do not fit Int32");
    return KI_OK;
}

}  // namespace

// filter(v -> abs(v) op t, x) and filter(v -> abs2(v) op t, x) (compact_map.cu).
__attribute__((visibility("hidden"))) int ki_compact_mapped(ki_ctx* ctx, int map, int pred, int dtype, const void* d_x,
                                                            size_t n, const void* h_thr, void* d_out_vals,
                                                            int32_t* d_out_idx, int64_t index_base, uint64_t* d_count,
                                                            cudaStream_t s);
