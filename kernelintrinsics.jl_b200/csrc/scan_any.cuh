// scan_any.cuh -- device-wide inclusive or exclusive scan for Base's +, *, max, min, |, &, xor over
// Int8 ... UInt64, Float32 and Float64 (Base.cumsum / cumprod / accumulate(op, x; init)).  The
// kernel and its launch are templates; scan_any*.cu instantiate them an operator family per file.
//
// The pipeline of scan.cu (one persistent CTA per SM, 31 work warps + 1 look warp, tiles taken in
// ticket order, 1-D TMA bulk staging, decoupled lookback of tile k-1 while tile k is summed, second
// pass from L2), generalised over the element type T and the operator:
//   * a tile is 124 KiB of input: 15872 elements of 8 bytes ... 126976 of 1 byte; a row is 32 lanes
//     x one 16-byte vector (2 to 16 elements per lane), a warp owns 8 rows;
//   * values are accumulated in Traits<T, Op>::A (ki/ops.cuh: 64-bit integers for sums and products
//     of smaller integers, Float64 for Float32 sums and products) and written as Traits<T, Op>::R
//     (Int64/UInt64 when widened, Float32 for Float32, T otherwise), as Base.cumsum/cumprod do;
//   * tile aggregates and prefixes ride in the status words when they fit (4-byte values, 8-byte
//     integers within 61 bits) and otherwise travel through the lookback's side arrays
//     (decoupled_lookback_any in ki/lookback.cuh).
// The Int64 + scan keeps its own kernel (scan.cu), whose values travel packed in the status words.
//
// Exclusive scans write op(init, x[1..i-1]) at i (init at the first element); inclusive scans
// op(init, x[1..i]).  Float sums are deterministic up to the order in which lookback windows find
// their predecessors, i.e. to Float64 rounding before the final Float32 rounding.
#pragma once

#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"
#include "ki/ops.cuh"

#include <limits>

// rows x cols, row r of the input at r*ld_in elements and of the output at r*ld_out (rows = 1: a
// plain scan of cols elements; the leading dimensions are then ignored).
struct ScanShape {
    size_t rows, cols, ld_in, ld_out;
};

namespace {

#ifndef KI_SCAN_ANY_SMALL_BATCH
#define KI_SCAN_ANY_SMALL_BATCH 2
#endif
constexpr int kWorkWarps = 31;
constexpr int kLookWarp = kWorkWarps;
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = kWorkThreads + 32;
// Rows per warp for 2- and 1-byte elements (8 for wider ones).  Measured at 2^28-2^30 (fraction of
// the copy peak, UInt8 cumsum / Int8 accumulate(max) / UInt8 accumulate(|)): 2 rows 0.41 / 0.25 /
// 0.35, 4 rows 0.42 / 0.31 / 0.46, 8 rows 0.41 / 0.34 / 0.52, 12 rows 0.39 / 0.33 / 0.48, 14 rows
// 0.38 / 0.34 / 0.50: the tile size is not what holds these back.
// Two 16-byte vectors per lane and step for 4- and 8-byte elements (one warp scan per 2*kE
// elements a lane, lanes 32 bytes apart) was slower everywhere at 2^28: Float32 cumsum 0.76 -> 0.66,
// Int32 -> Int64 cumsum 0.84 -> 0.68, Float64 cumsum 0.72 -> 0.69, Int32 xor 0.89 -> 0.81.
// Lane-wise (SWAR) scans load all 8 rows of a warp's span before scanning them.  With the packed
// lane totals that spills 16-36 bytes in the 1-byte instances; loading 4 rows at a time removes
// most of it but is slower (UInt8 | 0.646 -> 0.638, Int8 max 0.571 -> 0.547, Int16 | 0.846 ->
// 0.798, Int16 max 0.846 -> 0.776): the loads in flight matter more than the spills.
#ifndef KI_SCAN_ANY_SWAR_ALLROWS
#define KI_SCAN_ANY_SWAR_ALLROWS 1
#endif
#ifndef KI_SCAN_ANY_PACK_F32
#define KI_SCAN_ANY_PACK_F32 1
#endif
#ifndef KI_SCAN_ANY_PACK_TOTALS
#define KI_SCAN_ANY_PACK_TOTALS 1
#endif
// How tile values ride in the status words (ki/lookback.cuh).  Float32 sums and products accumulate
// in Float64 and are rounded to Float32 on output: one word, 3 mantissa bits dropped.  Everything
// else: one word when the value fits (the side arrays behind a fence otherwise).
// KI_SCAN_ANY_PAIR=1 puts 8-byte values other than integer sums in word pairs instead (no side
// arrays, no fence, two loads per tile and window).  Measured at 2^27 (fraction of the copy peak,
// one word -> pairs): Float64 cumsum 0.70 -> 0.71, Float64 cumprod 0.70 -> 0.71, Int64 xor of random
// values 0.68 -> 0.70, but where the values mostly fit 61 bits the second load costs: UInt64 | 0.79
// -> 0.70, Int64 cumprod 0.69 -> 0.63, Int32 cumprod into Int64 0.73 -> 0.69.  The Float64 scans are
// not held back by their lookback, so pairs stay off.
#ifndef KI_SCAN_ANY_PAIR
#define KI_SCAN_ANY_PAIR 0
#endif
#ifndef KI_SCAN_ANY_INVERSE
#define KI_SCAN_ANY_INVERSE 1
#endif
#ifndef KI_SCAN_ANY_IDEMPOTENT
#define KI_SCAN_ANY_IDEMPOTENT 1
#endif
template <class Op>
constexpr bool idempotent() {
    return KI_SCAN_ANY_IDEMPOTENT && (std::is_same<Op, ki::JMax>::value || std::is_same<Op, ki::JMin>::value ||
                                      std::is_same<Op, ki::JOr>::value || std::is_same<Op, ki::JAnd>::value);
}
// Inclusive warp scan (ki::warpreduce).  For idempotent operators no lane test is needed: where the
// source lane would be below lane 0, __shfl_up_sync returns the caller's own value, and op(v, v) = v.
// At 2^28 (fraction of the copy peak, with the lane test -> without): Float32 accumulate(max) 0.623
// -> 0.672, (min) 0.622 -> 0.669, Float64 max 0.515 -> 0.532, Int8 max 0.571 -> 0.581, UInt8 | 0.634
// -> 0.649; Int32 max and & and Int16 max unchanged (0.84-0.90); results identical.
template <class Op, class A, class F>
__device__ __forceinline__ A warp_scan(A v, F op) {
    if constexpr (idempotent<Op>()) {
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) v = op(ki::shfl<ki::Dir::Up>(v, off), v);
        return v;
    } else {
        return ki::warpreduce(v, op);
    }
}
// Operators whose lanes' exclusive prefix follows from the inclusive one and the lane's own total
// exactly (wrapping integer +, xor): no shuffle for it.  At 2^27 (fraction of the copy peak, with
// the shuffle -> without): UInt8 cumsum into UInt64 0.74 -> 0.77, Int64 + of values beyond 61 bits
// 0.706 -> 0.717, Int32 xor 0.846 -> 0.855, Int32 cumsum into Int64 0.81 -> 0.80; results identical.
template <class A, class Op>
constexpr bool has_inverse() {
    return KI_SCAN_ANY_INVERSE && std::is_integral<A>::value &&
           (std::is_same<Op, ki::JAdd>::value || std::is_same<Op, ki::JXor>::value);
}
template <class Op, class A>
__device__ __forceinline__ A exclusive_from(A inc, A tot) {
    using U = typename std::make_unsigned<A>::type;
    if constexpr (std::is_same<Op, ki::JXor>::value) return (A)((U)inc ^ (U)tot);
    else return (A)((U)inc - (U)tot);
}
template <class T, class Op>
constexpr bool status_lossy() {
    using A = typename ki::Traits<T, Op>::A;
    return KI_SCAN_ANY_PACK_F32 && std::is_same<T, float>::value && std::is_same<A, double>::value;
}
template <class T, class Op>
constexpr bool status_pair() {
    using A = typename ki::Traits<T, Op>::A;
    return KI_SCAN_ANY_PAIR && sizeof(A) == 8 && !status_lossy<T, Op>() &&
           !(std::is_integral<A>::value && std::is_same<Op, ki::JAdd>::value);
}
#ifndef KI_SCAN_ANY_ROWS_2B
#define KI_SCAN_ANY_ROWS_2B 8
#endif
#ifndef KI_SCAN_ANY_ROWS_1B
#define KI_SCAN_ANY_ROWS_1B 8
#endif

template <class T>
struct Shape {
    static constexpr int kE = (int)(16 / sizeof(T));        // elements per lane per row
    static constexpr int kRow = 32 * kE;                     // elements per row
    static constexpr int kRows = sizeof(T) >= 4 ? 8 : sizeof(T) == 2 ? KI_SCAN_ANY_ROWS_2B : KI_SCAN_ANY_ROWS_1B;
    static constexpr int kSpan = kRows * kRow;               // elements per warp
    static constexpr int kTile = kWorkWarps * kSpan;          // elements per tile
    static constexpr size_t kTileBytes = (size_t)kWorkWarps * kRows * 32 * 16;  // 126976 B at 8 rows
};

// Widening scans of 1- and 2-byte elements (sums and products into 64 bits) give each lane 64 or
// 128 bytes of output per row: stored straight from registers, every 16-byte warp store would touch
// 32 lines.  Instead the results go through a per-warp 2 KiB shared-memory stage (16 or 32 lanes'
// outputs per round, swizzled so that neither the writes nor the read-back conflict on banks) and
// leave as 512 contiguous bytes per warp store.
#ifndef KI_SCAN_ANY_STAGE
#define KI_SCAN_ANY_STAGE 1
#endif
template <class T, class Op>
struct Stage {
    using R = typename ki::Traits<T, Op>::R;
    static constexpr int kLaneBytes = (int)(16 / sizeof(T)) * (int)sizeof(R);  // output bytes per lane and row
    static constexpr bool kOn = KI_SCAN_ANY_STAGE && sizeof(T) <= 2 && kLaneBytes >= 64;
    static constexpr int kWarpBytes = 2048;
    static constexpr int kChunks = kLaneBytes / 16;                       // 16-byte chunks per lane: 4 or 8
    static constexpr int kLanes = kOn ? kWarpBytes / kLaneBytes : 32;     // lanes per round: 32 or 16
    static constexpr int kRounds = 32 / kLanes;
    static constexpr size_t kBytes = kOn ? (size_t)kWorkWarps * kWarpBytes : 0;
    // chunk q of lane l of a round sits at l * kChunks + swz(q, l): 8 consecutive lanes writing the
    // same q, or 8 consecutive chunks read back, fall on 8 different 16-byte bank groups
    __device__ static __forceinline__ int swz(int q, int l) {
        return kChunks == 8 ? (q ^ (l & 7)) : ((q + (l >> 1)) & 3);
    }
};

// The identity the scan folds from.  For Float64 accumulation of + it is -0.0 (-0.0 + x is x for
// every x, while +0.0 + -0.0 is +0.0), so sums over negative zeros keep their sign as Base.cumsum's
// do; the other operators take their traits' identity.
template <class T, class Op>
__device__ __forceinline__ typename ki::Traits<T, Op>::A scan_identity() {
    using A = typename ki::Traits<T, Op>::A;
    if constexpr (std::is_floating_point<A>::value && std::is_same<Op, ki::JAdd>::value) return A(-0.0);
    else return ki::Traits<T, Op>::identity();
}

// One row of a lane-wise (SWAR) scan on its way out: the lane's four result words o0..o3, shifted
// by one element for an exclusive scan (the first element is then the running prefix, rb's lowest
// element), stored as one 16-byte vector when the tile is full and the output aligned, else element
// by element within count.
template <class SW, bool EXCL, class R>
__device__ __forceinline__ void swar_put(R* __restrict__ dst, int i, int count, bool vec, uint32_t o0, uint32_t o1,
                                         uint32_t o2, uint32_t o3, uint32_t rb) {
    constexpr int kTop = 32 - SW::kBits;
    if (EXCL) {
        o3 = (o3 << SW::kBits) | (o2 >> kTop);
        o2 = (o2 << SW::kBits) | (o1 >> kTop);
        o1 = (o1 << SW::kBits) | (o0 >> kTop);
        o0 = (o0 << SW::kBits) | (rb & SW::kMask);
    }
    if (vec) {
        __stcs(reinterpret_cast<uint4*>(dst + i), make_uint4(o0, o1, o2, o3));
    } else {
        const uint32_t o[4] = {o0, o1, o2, o3};
        constexpr int kPer = 32 / SW::kBits;  // elements per word
#pragma unroll
        for (int e = 0; e < 4 * kPer; ++e)
            if (i + e < count) dst[i + e] = (R)((o[e / kPer] >> (SW::kBits * (e % kPer))) & SW::kMask);
    }
}

// The input is rows x cols (rows = 1 for a plain scan): row r starts ld_in elements after row r-1
// in the input and ld_out after it in the output, and every row is a segment of its own, cut into
// tpr tiles; tile t is chunk t % tpr of row t / tpr.
struct AnyArgs {
    const void* in;
    void* out;
    size_t rows, cols, ld_in, ld_out, tpr;
    uint64_t init_bits;  // init in the accumulation type, as raw bits
    ki::TileStatus st;
    unsigned long long* ticket;
    uint32_t* status;
    uint64_t timeout_ns;
    int tma_in;   // input 16-byte aligned: full tiles come in by TMA and as 16-byte rows
    int vec_out;  // output 16-byte aligned: full tiles leave with 16-byte stores
};

template <class A>
struct PendingAny {
    unsigned long long t;
    A agg;
    A tile_excl;
    A warp_excl[kWorkWarps];
};

__device__ __forceinline__ void work_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkThreads) : "memory"); }

template <class T, class Op, bool EXCL>
__global__ void __launch_bounds__(kThreads, 1) scan_any_kernel(AnyArgs a) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    using S = Shape<T>;
    constexpr int kE = S::kE;
    constexpr bool kLossy = status_lossy<T, Op>();
    constexpr bool kPair = status_pair<T, Op>();
    const ki::OpFn<T, Op> op;
    const A id = scan_identity<T, Op>();
    const A init = ki::from_bits<A>(a.init_bits);
    const T* in = static_cast<const T*>(a.in);
    R* out = static_cast<R*>(a.out);

    extern __shared__ __align__(128) unsigned char smem_raw[];
    T* sb = reinterpret_cast<T*>(smem_raw);
    __shared__ __align__(8) uint64_t bar;
    __shared__ A warp_tot[kWorkWarps];
    __shared__ PendingAny<A> slot[2];
    __shared__ unsigned long long ticket;

    const int tid = threadIdx.x;
    const int w = tid >> 5;
    const unsigned lane = tid & 31;
    const uint64_t ntiles = (uint64_t)a.rows * a.tpr;
    struct Where {
        size_t in_off, out_off;  // element offsets of the tile's first element
        int count;               // elements in the tile
        bool head;               // first tile of its row
    };
    auto where = [&](uint64_t t) {
        size_t row = 0, chunk = (size_t)t;
        if (a.rows > 1) {  // (a plain scan is one row: no division)
            row = (size_t)(t / a.tpr);
            chunk = (size_t)(t - (uint64_t)row * a.tpr);
        }
        Where p;
        p.in_off = row * a.ld_in + chunk * (size_t)S::kTile;
        p.out_off = row * a.ld_out + chunk * (size_t)S::kTile;
        p.count = (int)min((size_t)S::kTile, a.cols - chunk * (size_t)S::kTile);
        p.head = chunk == 0;
        return p;
    };
    auto bulk_ok = [&](uint64_t t) { return a.tma_in && t < ntiles && where(t).count == S::kTile; };
    auto fetch = [&]() {
        const unsigned long long t = atomicAdd(a.ticket, 1ull);
        ticket = t;
        if (bulk_ok(t)) {
            ki::fence_proxy_async_smem();
            ki::mbar_arrive_expect_tx(&bar, (uint32_t)S::kTileBytes);
            ki::bulk_g2s_keep(sb, in + where(t).in_off, (uint32_t)S::kTileBytes, &bar);
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
    int cur = 0;
    while (true) {
        const uint64_t t_new = ticket;
        const bool new_valid = t_new < ntiles;
        if (!new_valid && !have_old) break;

        // ---- phase A: fold and publish tile k  ||  look back for tile k-1 ---------------------------
        if (w == kLookWarp) {
            if (have_old) {
                PendingAny<A>& o = slot[cur ^ 1];
                const A ex = ki::decoupled_lookback_any<1, kLossy, kPair>(a.st, o.t, o.agg, init, id, op, a.status,
                                                                   a.timeout_ns, where(o.t).head);
                if (lane == 0) o.tile_excl = ex;
            }
        } else if (new_valid) {
            const Where p = where(t_new);
            const size_t first = p.in_off;
            const int count = p.count;
            if (bulk_ok(t_new)) {
                if (!ki::mbar_wait_bounded(&bar, phase, a.status, a.timeout_ns))
                    ki::mbar_wait_bounded(&bar, phase, a.status, a.timeout_ns);  // never leave a copy in flight
                phase ^= 1u;
            } else {
                const T pad = ki::pad_value<T, Op>();
                for (int i = tid; i < S::kTile; i += kWorkThreads) sb[i] = (i < count) ? in[first + i] : pad;
                work_sync();
            }
            A s = id;
            if constexpr (ki::swar_on<T, Op>()) {
                using SW = ki::Swar<T, Op>;
                if constexpr (SW::kSplit) {
                    uint32_t ae = SW::kId, ao = SW::kId;
#pragma unroll
                    for (int j = 0; j < S::kRows; ++j)
                        SW::fold16(*reinterpret_cast<const uint4*>(sb + w * S::kSpan + S::kRow * j + kE * lane), ae, ao);
                    s = (A)(T)SW::fold_total(ae, ao);
                } else {
                    uint32_t acc = SW::kId;
#pragma unroll
                    for (int j = 0; j < S::kRows; ++j) {
                        const uint4 r = *reinterpret_cast<const uint4*>(sb + w * S::kSpan + S::kRow * j + kE * lane);
                        acc = SW::comb(acc, SW::comb(SW::comb(r.x, r.y), SW::comb(r.z, r.w)));
                    }
#pragma unroll
                    for (int sh = 16; sh >= SW::kBits; sh >>= 1)
                        acc = SW::comb(acc, (acc >> sh) | (SW::kId & ~(0xFFFFFFFFu >> sh)));
                    s = (A)(T)(acc & SW::kMask);
                }
            } else {
#pragma unroll
                for (int j = 0; j < S::kRows; ++j) {
                    ki::Packed16<T> v;
                    v.raw = *reinterpret_cast<const uint4*>(sb + w * S::kSpan + S::kRow * j + kE * lane);
#pragma unroll
                    for (int e = 0; e < kE; ++e) s = op(s, Tr::lift(v.get(e)));
                }
            }
            s = ki::warpfold(s, op);
            if (lane == 0) warp_tot[w] = s;
            work_sync();
            if (w == 0) {
                const A x = (lane < (unsigned)kWorkWarps) ? warp_tot[lane] : id;
                const A inc = warp_scan<Op>(x, op);
                A exc = __shfl_up_sync(0xffffffffu, inc, 1);
                if (lane == 0) exc = id;
                const A agg = __shfl_sync(0xffffffffu, inc, kWorkWarps - 1);
                PendingAny<A>& e = slot[cur];
                if (lane < (unsigned)kWorkWarps) e.warp_excl[lane] = exc;
                if (lane == 0) {
                    e.t = t_new;
                    e.agg = agg;
                    ki::publish_aggregate_any<kLossy, kPair>(a.st, t_new, agg, init, op, p.head);
                }
            }
        }
        __syncthreads();

        // ---- phase B: start tile k+1's load; finish tile k-1 -----------------------------------------
        if (tid == kLookWarp * 32 && new_valid) fetch();
        if (w < kWorkWarps && have_old) {
            const PendingAny<A>& o = slot[cur ^ 1];
            const Where p = where(o.t);
            const size_t first = p.in_off, out_first = p.out_off;
            const int count = p.count;
            const bool full = count == S::kTile;
            A carry = op(o.tile_excl, o.warp_excl[w]);
            const T pad = ki::pad_value<T, Op>();
            // rows in flight: all 8 for 4- and 8-byte elements; 1- and 2-byte elements take more
            // registers per row on the way out, so they go KI_SCAN_ANY_SMALL_BATCH rows at a time
            constexpr int kB = (sizeof(T) >= 4 || (ki::swar_on<T, Op>() && KI_SCAN_ANY_SWAR_ALLROWS)) ? S::kRows
                               : (KI_SCAN_ANY_SMALL_BATCH < S::kRows ? KI_SCAN_ANY_SMALL_BATCH : S::kRows);
            static_assert(S::kRows % kB == 0, "row batches");
#pragma unroll 1
            for (int j0 = 0; j0 < S::kRows; j0 += kB) {
            ki::Packed16<T> v[kB];
#pragma unroll
            for (int jj = 0; jj < kB; ++jj) {
                const int j = j0 + jj;
                const int i = w * S::kSpan + S::kRow * j + kE * (int)lane;
                if (full && a.tma_in) {
                    v[jj].raw = __ldcs(reinterpret_cast<const uint4*>(in + first + i));
                } else {
#pragma unroll
                    for (int e = 0; e < kE; ++e) v[jj].set(e, (i + e < count) ? in[first + i + e] : pad);
                }
            }
            constexpr bool kPacked = ki::swar_on<T, Op>() && KI_SCAN_ANY_PACK_TOTALS;
            if constexpr (kPacked) {
                // Lane-wise scans: the lane totals of G rows go into one word, one element lane per
                // row, so one warp scan with the lane-wise combine serves G rows (4 for bytes, 2 for
                // halfwords), and the rows' carries come from one prefix of the packed warp totals
                // (the operators here are commutative, so the combine order does not matter).
                // Against one warp scan per row, at 2^28 (fraction of the copy peak): UInt8 | 0.59 ->
                // 0.64, Int8 max 0.46 -> 0.57, UInt8 max 0.51 -> 0.59, Int16 | 0.78 -> 0.84, Int16 max
                // 0.75 -> 0.84, UInt16 max 0.77 -> 0.85, results identical.
                using SW = ki::Swar<T, Op>;
                using U = typename std::make_unsigned<T>::type;
                constexpr int kTop = 32 - SW::kBits;
                constexpr int G = 32 / SW::kBits;
                static_assert(kB % G == 0, "row groups");
#pragma unroll
                for (int g0 = 0; g0 < kB; g0 += G) {
                    uint32_t pe[G][4], po[G][4];  // the lanes' prefixes (split form: even and odd bytes)
                    uint32_t tw = 0;              // the lanes' totals, element lane r for row g0 + r
#pragma unroll
                    for (int r = 0; r < G; ++r) {
                        const uint4 raw = v[g0 + r].raw;
                        if constexpr (SW::kSplit) {
                            SW::prefix_split(raw.x, pe[r][0], po[r][0]);
                            SW::prefix_split(raw.y, pe[r][1], po[r][1]);
                            SW::prefix_split(raw.z, pe[r][2], po[r][2]);
                            SW::prefix_split(raw.w, pe[r][3], po[r][3]);
                            SW::chain(pe[r][1], po[r][1], po[r][0]);
                            SW::chain(pe[r][2], po[r][2], po[r][1]);
                            SW::chain(pe[r][3], po[r][3], po[r][2]);
                            tw |= (po[r][3] >> kTop) << (SW::kBits * r);
                        } else {
                            pe[r][0] = ki::swar_prefix<SW>(raw.x);
                            pe[r][1] = SW::comb(ki::swar_prefix<SW>(raw.y), SW::top(pe[r][0]));
                            pe[r][2] = SW::comb(ki::swar_prefix<SW>(raw.z), SW::top(pe[r][1]));
                            pe[r][3] = SW::comb(ki::swar_prefix<SW>(raw.w), SW::top(pe[r][2]));
                            tw |= (pe[r][3] >> kTop) << (SW::kBits * r);
                        }
                    }
                    uint32_t inc = tw;
#pragma unroll
                    for (int off = 1; off < 32; off <<= 1) {
                        const uint32_t x = __shfl_up_sync(0xffffffffu, inc, off);
                        if (idempotent<Op>() || (int)lane >= off) inc = SW::comb(x, inc);
                    }
                    uint32_t before = __shfl_up_sync(0xffffffffu, inc, 1);
                    if (lane == 0) before = SW::kId;
                    const uint32_t cb = SW::bcast((uint32_t)(U)carry);
                    // carry, then the warp totals of rows g0 .. g0 + r, in element lane r
                    const uint32_t cp = SW::comb(ki::swar_prefix<SW>(__shfl_sync(0xffffffffu, inc, 31)), cb);
                    // each row's running prefix at this lane: carry, the rows before, the lanes before
                    const uint32_t runs = SW::comb((cp << SW::kBits) | (cb & SW::kMask), before);
                    carry = (A)(T)(cp >> kTop);
#pragma unroll
                    for (int r = 0; r < G; ++r) {
                        const uint32_t rb = SW::spread(runs, r);
                        uint32_t o0, o1, o2, o3;
                        if constexpr (SW::kSplit) {
                            o0 = SW::join(SW::h(pe[r][0], rb), SW::h(po[r][0], rb));
                            o1 = SW::join(SW::h(pe[r][1], rb), SW::h(po[r][1], rb));
                            o2 = SW::join(SW::h(pe[r][2], rb), SW::h(po[r][2], rb));
                            o3 = SW::join(SW::h(pe[r][3], rb), SW::h(po[r][3], rb));
                        } else {
                            o0 = SW::comb(pe[r][0], rb), o1 = SW::comb(pe[r][1], rb);
                            o2 = SW::comb(pe[r][2], rb), o3 = SW::comb(pe[r][3], rb);
                        }
                        const int i = w * S::kSpan + S::kRow * (j0 + g0 + r) + kE * (int)lane;
                        swar_put<SW, EXCL>(out + out_first, i, count, full && a.vec_out, o0, o1, o2, o3, rb);
                    }
                }
            }
#pragma unroll
            for (int jj = 0; jj < (kPacked ? 0 : kB); ++jj) {
                const int j = j0 + jj;
                // the lane's total, the warp's scan of the totals, then the lane's prefixes again on
                // the way out (no per-element arrays: 16-byte lanes of 1-byte elements stay in registers)
                if constexpr (ki::swar_on<T, Op>()) {
                    using SW = ki::Swar<T, Op>;
                    constexpr int kTop = 32 - SW::kBits;  // shift of a word's last element
                    uint32_t o0, o1, o2, o3, rb;
                    A inc;
                    if constexpr (SW::kSplit) {
                        // byte max / min: the words stay split into even and odd bytes (the high bytes
                        // of halfwords) until the running prefix is in, then are joined once
                        uint32_t e0, d0, e1, d1, e2, d2, e3, d3;
                        SW::prefix_split(v[jj].raw.x, e0, d0);
                        SW::prefix_split(v[jj].raw.y, e1, d1);
                        SW::prefix_split(v[jj].raw.z, e2, d2);
                        SW::prefix_split(v[jj].raw.w, e3, d3);
                        SW::chain(e1, d1, d0);
                        SW::chain(e2, d2, d1);
                        SW::chain(e3, d3, d2);
                        inc = warp_scan<Op>((A)(T)(d3 >> kTop), op);
                        A before = __shfl_up_sync(0xffffffffu, inc, 1);
                        if (lane == 0) before = id;
                        const A run = op(carry, before);
                        rb = SW::bcast((uint32_t)(typename std::make_unsigned<T>::type)run);
                        o0 = SW::join(SW::h(e0, rb), SW::h(d0, rb));
                        o1 = SW::join(SW::h(e1, rb), SW::h(d1, rb));
                        o2 = SW::join(SW::h(e2, rb), SW::h(d2, rb));
                        o3 = SW::join(SW::h(e3, rb), SW::h(d3, rb));
                    } else {
                        uint32_t y0 = ki::swar_prefix<SW>(v[jj].raw.x), y1 = ki::swar_prefix<SW>(v[jj].raw.y);
                        uint32_t y2 = ki::swar_prefix<SW>(v[jj].raw.z), y3 = ki::swar_prefix<SW>(v[jj].raw.w);
                        y1 = SW::comb(y1, SW::top(y0));
                        y2 = SW::comb(y2, SW::top(y1));
                        y3 = SW::comb(y3, SW::top(y2));
                        inc = warp_scan<Op>((A)(T)(y3 >> kTop), op);
                        A before = __shfl_up_sync(0xffffffffu, inc, 1);
                        if (lane == 0) before = id;
                        const A run = op(carry, before);
                        rb = SW::bcast((uint32_t)(typename std::make_unsigned<T>::type)run);
                        o0 = SW::comb(y0, rb), o1 = SW::comb(y1, rb), o2 = SW::comb(y2, rb), o3 = SW::comb(y3, rb);
                    }
                    const int i = w * S::kSpan + S::kRow * j + kE * (int)lane;
                    swar_put<SW, EXCL>(out + out_first, i, count, full && a.vec_out, o0, o1, o2, o3, rb);
                    carry = op(carry, __shfl_sync(0xffffffffu, inc, 31));
                    continue;
                }
                A tot = Tr::lift(v[jj].get(0));
#pragma unroll
                for (int e = 1; e < kE; ++e) tot = op(tot, Tr::lift(v[jj].get(e)));
                const A inc = warp_scan<Op>(tot, op);
                A before;
                if constexpr (has_inverse<A, Op>()) {
                    before = exclusive_from<Op>(inc, tot);
                } else {
                    before = __shfl_up_sync(0xffffffffu, inc, 1);
                    if (lane == 0) before = id;
                }
                A run = op(carry, before);
                const int i = w * S::kSpan + S::kRow * j + kE * (int)lane;
                if constexpr (Stage<T, Op>::kOn) {
                    if (full && a.vec_out) {
                        using St = Stage<T, Op>;
                        constexpr int kPer = (int)(16 / sizeof(R));
                        uint4* stg = reinterpret_cast<uint4*>(smem_raw + S::kTileBytes) + (size_t)w * (St::kWarpBytes / 16);
                        R* orow = out + out_first + (size_t)(w * S::kSpan + S::kRow * j);
#pragma unroll 1
                        for (int rd = 0; rd < St::kRounds; ++rd) {
                            if ((int)lane / St::kLanes == rd) {
                                const int ll = (int)lane % St::kLanes;
#pragma unroll
                                for (int q = 0; q < St::kChunks; ++q) {
                                    alignas(16) R r[kPer];
#pragma unroll
                                    for (int p = 0; p < kPer; ++p) {
                                        const A x = Tr::lift(v[jj].get(q * kPer + p));
                                        if (EXCL) {
                                            r[p] = Tr::lower(run);
                                            run = op(run, x);
                                        } else {
                                            run = op(run, x);
                                            r[p] = Tr::lower(run);
                                        }
                                    }
                                    stg[ll * St::kChunks + St::swz(q, ll)] = *reinterpret_cast<const uint4*>(r);
                                }
                            }
                            __syncwarp();
                            uint4* g = reinterpret_cast<uint4*>(orow + (size_t)rd * St::kLanes * kE);
#pragma unroll
                            for (int c = 0; c < St::kWarpBytes / 16 / 32; ++c) {
                                const int gi = c * 32 + (int)lane;
                                const int ls = gi / St::kChunks, q = gi % St::kChunks;
                                __stcs(g + gi, stg[ls * St::kChunks + St::swz(q, ls)]);
                            }
                            __syncwarp();
                        }
                        carry = op(carry, __shfl_sync(0xffffffffu, inc, 31));
                        continue;
                    }
                }
                if (full && a.vec_out) {
                    constexpr int kPer = (int)(16 / sizeof(R));  // results per 16-byte store
                    constexpr int kStores = kE / kPer;
#pragma unroll
                    for (int q = 0; q < kStores; ++q) {
                        alignas(16) R r[kPer];
#pragma unroll
                        for (int p = 0; p < kPer; ++p) {
                            const A x = Tr::lift(v[jj].get(q * kPer + p));
                            if (EXCL) {
                                r[p] = Tr::lower(run);
                                run = op(run, x);
                            } else {
                                run = op(run, x);
                                r[p] = Tr::lower(run);
                            }
                        }
                        __stcs(reinterpret_cast<uint4*>(out + out_first + i) + q, *reinterpret_cast<const uint4*>(r));
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < kE; ++e) {
                        const A x = Tr::lift(v[jj].get(e));
                        R r;
                        if (EXCL) {
                            r = Tr::lower(run);
                            run = op(run, x);
                        } else {
                            run = op(run, x);
                            r = Tr::lower(run);
                        }
                        if (i + e < count) out[out_first + i + e] = r;
                    }
                }
                carry = op(carry, __shfl_sync(0xffffffffu, inc, 31));
            }
            }
        }
        __syncthreads();
        have_old = new_valid;
        cur ^= 1;
    }
}

// Short rows (at most kShortRowBytes of input): one warp per row, 32 lanes x one 16-byte vector
// per step (the next step's vector loaded before this one is scanned), the carry passed along the
// row; no tile status, no lookback.
constexpr size_t kShortRowBytes = 32768;
constexpr int kRowThreads = 256;

template <class T, class Op, bool EXCL>
__global__ void __launch_bounds__(kRowThreads) scan_rows_warp_kernel(const T* __restrict__ in,
                                                                     typename ki::Traits<T, Op>::R* __restrict__ out,
                                                                     size_t rows, size_t cols, size_t ld_in,
                                                                     size_t ld_out, uint64_t init_bits, int vec_in,
                                                                     int vec_out) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    constexpr int kE = (int)(16 / sizeof(T));
    constexpr int kRow = 32 * kE;
    const ki::OpFn<T, Op> op;
    const A id = scan_identity<T, Op>();
    const A init = ki::from_bits<A>(init_bits);
    const T pad = ki::pad_value<T, Op>();
    const unsigned lane = threadIdx.x & 31;
    const size_t nwarps = ((size_t)gridDim.x * kRowThreads) >> 5;
    auto load = [&](const T* x, size_t c0) {
        ki::Packed16<T> v;
        const size_t i = c0 + (size_t)kE * lane;
        if (vec_in && c0 + kRow <= cols) {
            v.raw = __ldcs(reinterpret_cast<const uint4*>(x + i));
        } else {
#pragma unroll
            for (int e = 0; e < kE; ++e) v.set(e, (i + e < cols) ? x[i + e] : pad);
        }
        return v;
    };
    for (size_t row = ((size_t)blockIdx.x * kRowThreads + threadIdx.x) >> 5; row < rows; row += nwarps) {
        const T* x = in + row * ld_in;
        R* y = out + row * ld_out;
        A carry = init;
        ki::Packed16<T> next = load(x, 0);
        for (size_t c0 = 0; c0 < cols; c0 += kRow) {
            const ki::Packed16<T> v = next;
            if (c0 + kRow < cols) next = load(x, c0 + kRow);
            A tot = Tr::lift(v.get(0));
#pragma unroll
            for (int e = 1; e < kE; ++e) tot = op(tot, Tr::lift(v.get(e)));
            const A inc = warp_scan<Op>(tot, op);
            A before = __shfl_up_sync(0xffffffffu, inc, 1);
            if (lane == 0) before = id;
            A run = op(carry, before);
            const size_t i = c0 + (size_t)kE * lane;
            if (vec_out && c0 + kRow <= cols) {
                constexpr int kPer = (int)(16 / sizeof(R));
#pragma unroll
                for (int q = 0; q < kE / kPer; ++q) {
                    alignas(16) R r[kPer];
#pragma unroll
                    for (int p = 0; p < kPer; ++p) {
                        const A xv = Tr::lift(v.get(q * kPer + p));
                        if (EXCL) {
                            r[p] = Tr::lower(run);
                            run = op(run, xv);
                        } else {
                            run = op(run, xv);
                            r[p] = Tr::lower(run);
                        }
                    }
                    __stcs(reinterpret_cast<uint4*>(y + i) + q, *reinterpret_cast<const uint4*>(r));
                }
            } else {
#pragma unroll
                for (int e = 0; e < kE; ++e) {
                    const A xv = Tr::lift(v.get(e));
                    R r;
                    if (EXCL) {
                        r = Tr::lower(run);
                        run = op(run, xv);
                    } else {
                        run = op(run, xv);
                        r = Tr::lower(run);
                    }
                    if (i + e < cols) y[i + e] = r;
                }
            }
            carry = op(carry, __shfl_sync(0xffffffffu, inc, 31));
        }
    }
}

// init: a host value of the result type, converted to the accumulation type; else the identity.
template <class T, class Op>
typename ki::Traits<T, Op>::A init_value(const void* h_init) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    if (h_init) {
        R r;
        memcpy(&r, h_init, sizeof(R));
        if constexpr (std::is_same<Op, ki::JAdd>::value || std::is_same<Op, ki::JMul>::value) return (A)r;
        else return Tr::lift(r);
    } else if constexpr (std::is_same<Op, ki::JAdd>::value) {
        return A(0);
    } else if constexpr (std::is_same<Op, ki::JMul>::value) {
        return A(1);
    } else if constexpr (ki::IsBitwise<Op>::value) {
        return Tr::identity();
    } else if constexpr (std::is_floating_point<T>::value) {
        return Tr::lift(std::is_same<Op, ki::JMax>::value ? -std::numeric_limits<T>::infinity()
                                                          : std::numeric_limits<T>::infinity());
    } else {
        return std::is_same<Op, ki::JMax>::value ? std::numeric_limits<A>::lowest() : std::numeric_limits<A>::max();
    }
}

template <class T, class Op>
int scan_launch(ki_ctx* ctx, bool excl, const void* d_in, void* d_out, const ScanShape& sh, const void* h_init,
                cudaStream_t s) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    using S = Shape<T>;
    if (!ki::aligned(d_in, sizeof(T)) || !ki::aligned(d_out, sizeof(R)))
        return ki::set_error(ctx, KI_ERR_ARG, "scan: misaligned input or output");
    const size_t rows = sh.rows, cols = sh.cols;
    const size_t ld_in = rows > 1 ? sh.ld_in : cols, ld_out = rows > 1 ? sh.ld_out : cols;
    const uintptr_t i0 = (uintptr_t)d_in, o0 = (uintptr_t)d_out;
    const uintptr_t ib = ((rows - 1) * ld_in + cols) * sizeof(T), ob = ((rows - 1) * ld_out + cols) * sizeof(R);
    const bool in_place = i0 == o0 && sizeof(T) == sizeof(R) && ld_in == ld_out;
    if (!in_place && i0 < o0 + ob && o0 < i0 + ib)
        return ki::set_error(ctx, KI_ERR_ARG, "scan: input and output overlap (only an exact in-place scan is allowed)");
    A init = init_value<T, Op>(h_init);
    // an inclusive float cumsum without init starts from -0.0, the identity: out[1] is x[1], sign
    // included (an exclusive one writes its init, +0.0, first)
    if constexpr (std::is_floating_point<A>::value && std::is_same<Op, ki::JAdd>::value)
        if (!h_init && !excl) init = A(-0.0);
    uint64_t init_bits = 0;
    memcpy(&init_bits, &init, sizeof(A));
    const int vec_in = ki::aligned(d_in, 16) && (rows == 1 || (ld_in * sizeof(T)) % 16 == 0);
    const int vec_out = ki::aligned(d_out, 16) && (rows == 1 || (ld_out * sizeof(R)) % 16 == 0);
    if (rows > 1 && cols * sizeof(T) <= kShortRowBytes) {
        size_t blocks = (rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
        const size_t cap = (size_t)ctx->sm_count * (2048 / kRowThreads);
        if (blocks > cap) blocks = cap;
        const T* x = static_cast<const T*>(d_in);
        R* y = static_cast<R*>(d_out);
        if (excl)
            scan_rows_warp_kernel<T, Op, true><<<(unsigned)blocks, kRowThreads, 0, s>>>(x, y, rows, cols, ld_in, ld_out,
                                                                                      init_bits, vec_in, vec_out);
        else
            scan_rows_warp_kernel<T, Op, false><<<(unsigned)blocks, kRowThreads, 0, s>>>(x, y, rows, cols, ld_in, ld_out,
                                                                                       init_bits, vec_in, vec_out);
        return ki::check_launch(ctx, "scan_rows_warp_kernel launch");
    }
    const size_t tpr = (cols + S::kTile - 1) / S::kTile;
    const size_t ntiles = rows * tpr;
    const size_t words_off = 256;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_SCAN_ANY, words_off + ntiles * 24, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    // status words: one per tile, or two per tile when values ride in pairs (the region's next 8
    // bytes per tile, otherwise the aggregates' side array)
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, words_off + ntiles * (status_pair<T, Op>() ? 16 : 8), s));
    AnyArgs a;
    a.in = d_in;
    a.out = d_out;
    a.rows = rows;
    a.cols = cols;
    a.ld_in = ld_in;
    a.ld_out = ld_out;
    a.tpr = tpr;
    a.init_bits = init_bits;
    a.st.words = reinterpret_cast<uint64_t*>(b + words_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + words_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + words_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.tma_in = vec_in;
    a.vec_out = vec_out;
    size_t grid = (size_t)ctx->sm_count;
    if (grid > ntiles) grid = ntiles;
    if (excl) {
        KI_CUDA(ctx, cudaFuncSetAttribute(scan_any_kernel<T, Op, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(S::kTileBytes + Stage<T, Op>::kBytes)));
        scan_any_kernel<T, Op, true><<<(unsigned)grid, kThreads, S::kTileBytes + Stage<T, Op>::kBytes, s>>>(a);
    } else {
        KI_CUDA(ctx, cudaFuncSetAttribute(scan_any_kernel<T, Op, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(S::kTileBytes + Stage<T, Op>::kBytes)));
        scan_any_kernel<T, Op, false><<<(unsigned)grid, kThreads, S::kTileBytes + Stage<T, Op>::kBytes, s>>>(a);
    }
    return ki::check_launch(ctx, "scan_any_kernel launch");
}

template <class Op>
int scan_op(ki_ctx* ctx, int dtype, bool excl, const void* d_in, void* d_out, const ScanShape& sh, const void* h_init,
            cudaStream_t s) {
    constexpr int kBad = -1000;
    const int rc = ki::with_dtype(dtype, kBad, [&](auto tag) -> int {
        using T = decltype(tag);
        if constexpr (ki::op_takes<T, Op>()) return scan_launch<T, Op>(ctx, excl, d_in, d_out, sh, h_init, s);
        else return kBad;
    });
    if (rc == kBad) return ki::set_error(ctx, KI_ERR_ARG, "scan: the operator does not take this element type");
    return rc;
}

}  // namespace

// One per operator, defined in scan_any*.cu.
#define KI_SCAN_ANY_ENTRY(name)                                                                                \
    __attribute__((visibility("hidden"))) int name(ki_ctx* ctx, int dtype, bool excl, const void* d_in, void* d_out, \
                                                   const ScanShape& sh, const void* h_init, cudaStream_t s)
KI_SCAN_ANY_ENTRY(ki_scan_any_add);
KI_SCAN_ANY_ENTRY(ki_scan_any_mul);
KI_SCAN_ANY_ENTRY(ki_scan_any_max);
KI_SCAN_ANY_ENTRY(ki_scan_any_min);
KI_SCAN_ANY_ENTRY(ki_scan_any_or);
KI_SCAN_ANY_ENTRY(ki_scan_any_and);
KI_SCAN_ANY_ENTRY(ki_scan_any_xor);
