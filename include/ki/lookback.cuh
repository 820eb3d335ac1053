// ki/lookback.cuh -- decoupled lookback over per-tile status words, and 1-D TMA bulk helpers.
//
// Tile status, one 64-bit word per tile (reset to 0 before each call):
//   bits 0-1  state: 0 = nothing published, 1 = aggregate published (A), 2 = inclusive prefix (P)
//   bit  2    wide: the value did not fit and lives in aggs[t] (A) or incls[t] (P)
//   bits 3-63 the value as a 61-bit two's-complement integer (when not wide)
// A packed word is published with one st.release.gpu and read with one ld.acquire.gpu, so looking
// back over a window of 32 tiles costs one round trip to L2.  A value outside the 61-bit range is
// first written to its side array with a plain store, then the word (state | wide) is published
// with st.release.gpu; a reader that acquires such a word loads the value with ld.relaxed.gpu.
// These are the @access store / load defaults of the reference (src/macros.jl:259-275 ->
// ext/CUDA/scopes_ordering.jl:89-193).
//
// Every wait is bounded by %globaltimer: when it runs out the warp latches KI_DEV_TIMEOUT in the
// status word it was given and carries on with what it has, so the grid always finishes.
#pragma once

#include <cstdint>
#include <cstring>

#include "intrinsics.cuh"
#include "status.h"

// Sleep between re-reads of a window that still has unpublished tiles (doubles up to the max).
#ifndef KI_LOOKBACK_MIN_SLEEP_NS
#define KI_LOOKBACK_MIN_SLEEP_NS 32
#endif
#ifndef KI_LOOKBACK_MAX_SLEEP_NS
#define KI_LOOKBACK_MAX_SLEEP_NS 512
#endif

namespace ki {

constexpr uint64_t kFlagNone = 0, kFlagAgg = 1, kFlagPrefix = 2, kFlagWide = 4;

struct TileStatus {
    uint64_t* words;
    int64_t* aggs;
    int64_t* incls;
};

__device__ __forceinline__ bool fits61(int64_t v) { return v >= -(1ll << 60) && v < (1ll << 60); }

__device__ __forceinline__ void publish(TileStatus st, uint64_t t, uint64_t state, int64_t v) {
    if (fits61(v)) {
        store<Order::Release, Scope::Device>(&st.words[t], ((uint64_t)v << 3) | state);
    } else {
        (state == kFlagPrefix ? st.incls : st.aggs)[t] = v;
        store<Order::Release, Scope::Device>(&st.words[t], kFlagWide | state);
    }
}

// Run by all 32 lanes of one warp, after publish_aggregate(t).  Looks back over predecessors until
// an inclusive prefix is found, publishes tile t's inclusive prefix and returns the exclusive prefix
// of tile t (including `seed`).  Sums wrap around (two's complement).
//
// The window is 32*K tiles: lane l reads the K words of tiles end-(l*K) .. end-(l*K+K-1) with
// independent ld.relaxed.gpu loads, so a whole window costs one round trip (acquire loads would be
// performed one after another).  Packed words carry their value, so nothing else is read; a wide
// value is read from its side array after a fence.acq_rel.gpu, which with the relaxed load of its
// word is the fence form of an acquire (@access Relaxed + @fence).  Throughput of a lookback
// chain is bounded by window / round trip, hence the wide window.
//
// The caller publishes the tile's aggregate first (publish_aggregate), as soon as its data has
// landed, and may do other work before looking back: a tile's aggregate must never wait behind its
// owner's other work, or owners end up waiting on one another.
__device__ __forceinline__ void publish_aggregate(TileStatus st, uint64_t t, int64_t agg, int64_t seed) {
    if (t == 0) publish(st, 0, kFlagPrefix, wrap_add(seed, agg));
    else publish(st, t, kFlagAgg, agg);
}

template <int K>
__device__ __forceinline__ int64_t decoupled_lookback(TileStatus st, uint64_t t, int64_t agg, int64_t seed,
                                                      uint32_t* status, uint64_t timeout_ns) {
    const unsigned lane = lane0();
    if (t == 0) return seed;
    int64_t excl = 0;
    long long end = (long long)t - 1;  // nearest tile of the current window
    uint64_t t_start = 0;
    bool timed_out = false;
    unsigned backoff = KI_LOOKBACK_MIN_SLEEP_NS;
    while (true) {
        uint64_t w[K];
        int first_p, first_zero;  // lane-local positions (K = none)
        int pos_p, pos_zero;      // window positions l*K+k of the first P / unpublished word
        while (true) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const long long idx = end - (long long)(lane * K + k);
                w[k] = (idx >= 0) ? load<Order::Relaxed, Scope::Device>(&st.words[idx]) : kFlagPrefix;
            }
            first_p = K;
            first_zero = K;
#pragma unroll
            for (int k = K - 1; k >= 0; --k) {
                if ((w[k] & 3) == kFlagPrefix) first_p = k;
                if ((w[k] & 3) == kFlagNone) first_zero = k;
            }
            const unsigned pm = __ballot_sync(0xffffffffu, first_p < K);
            const unsigned zm = __ballot_sync(0xffffffffu, first_zero < K);
            const int lp = pm ? __ffs(pm) - 1 : 32, lz = zm ? __ffs(zm) - 1 : 32;
            pos_p = (lp < 32) ? lp * K + __shfl_sync(0xffffffffu, first_p, lp) : 32 * K;
            pos_zero = (lz < 32) ? lz * K + __shfl_sync(0xffffffffu, first_zero, lz) : 32 * K;
            if (pos_zero > pos_p || (pos_zero == 32 * K && pos_p == 32 * K)) break;  // nothing missing before the P
            const uint64_t now = globaltimer_ns();
            if (t_start == 0) t_start = now;
            timed_out = __shfl_sync(0xffffffffu, (int)(now - t_start > timeout_ns), 0) != 0;
            if (timed_out) break;
            __nanosleep(backoff);  // the window re-read is 32*K loads: back off to spare L2
            if (backoff < KI_LOOKBACK_MAX_SLEEP_NS) backoff <<= 1;
        }
        if (timed_out) {
            if (lane == 0) atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
            break;
        }
        // sum the words at positions <= pos_p (all of the window when it holds no P)
        bool any_wide = false;
        int64_t v = 0;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int p = (int)lane * K + k;
            if (p <= pos_p && p < 32 * K) {
                if (w[k] & kFlagWide) any_wide = true;
                else v = wrap_add(v, (int64_t)w[k] >> 3);
            }
        }
        if (__any_sync(0xffffffffu, any_wide)) {
            fence<Scope::Device, Order::AcqRel>();
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int p = (int)lane * K + k;
                const long long idx = end - p;
                if (p <= pos_p && p < 32 * K && (w[k] & kFlagWide)) {
                    const int64_t x = ((w[k] & 3) == kFlagPrefix) ? load<Order::Relaxed, Scope::Device>(&st.incls[idx])
                                                                  : load<Order::Relaxed, Scope::Device>(&st.aggs[idx]);
                    v = wrap_add(v, x);
                }
            }
        }
        excl = wrap_add(excl, warpfold(v, WrapAdd{}));
        if (pos_p < 32 * K) break;
        end -= 32 * K;
    }
    if (lane == 0) publish(st, t, kFlagPrefix, wrap_add(excl, agg));
    return excl;
}

// ---------------------------------------------------------------------------------------------
// Lookback for any operator and value type of at most 8 bytes (the generic scan).  A value rides in
// its status word when it fits, as in decoupled_lookback: 4-byte values always (bits 32-63),
// 8-byte integers when their two's-complement value fits 61 bits (bits 3-63).  Anything else
// (every Float64, large 64-bit integers) lives in the side arrays (aggs for aggregates, incls for
// inclusive prefixes, as raw bits) with the wide bit set in its status word; a fence.acq_rel.gpu
// orders those value loads after the status loads.  With PAIR every value rides in two status words
// instead (publish_any), so a window is one round trip to L2 for any 8-byte value.  `op` must be associative and commutative
// (Base + on integers, max, min; Float64 + up to rounding).
// ---------------------------------------------------------------------------------------------
template <class A>
__device__ __forceinline__ uint64_t to_bits(A v) {
    uint64_t b = 0;
    memcpy(&b, &v, sizeof(A));
    return b;
}
template <class A>
__device__ __forceinline__ A from_bits(uint64_t b) {
    A v;
    memcpy(&v, &b, sizeof(A));
    return v;
}

// Packing of a value into a status word (state in bits 0-1, wide bit 2).  LOSSY (a Float64 that is
// rounded to Float32 at the end anyway): the double rides in the word with its 3 lowest mantissa
// bits dropped, a relative change below 2^-49.
template <bool LOSSY = false, class A>
__device__ __forceinline__ bool pack_value(A v, uint64_t& word_bits) {
    if constexpr (LOSSY && std::is_same<A, double>::value) {
        word_bits = to_bits(v) & ~(uint64_t)7;
        return true;
    } else if constexpr (sizeof(A) == 4) {
        word_bits = to_bits(v) << 32;
        return true;
    } else if constexpr (std::is_integral<A>::value) {
        const int64_t s = (int64_t)to_bits(v);
        if (!fits61(s)) return false;
        word_bits = (uint64_t)s << 3;
        return true;
    } else {
        return false;
    }
}
template <class A, bool LOSSY = false>
__device__ __forceinline__ A unpack_value(uint64_t w) {
    if constexpr (LOSSY && std::is_same<A, double>::value) return from_bits<A>(w & ~(uint64_t)7);
    else if constexpr (sizeof(A) == 4) return from_bits<A>(w >> 32);
    else return from_bits<A>((uint64_t)((int64_t)w >> 3));
}

// PAIR: an 8-byte value rides in two status words, words[2t] (its high 32 bits) and words[2t + 1]
// (its low 32 bits), each beside the state; a tile's states only move none -> aggregate -> prefix
// and each state has one value, so two words that show the same state hold one value, and a pair
// caught between two publishes (states differ) reads as not ready.  No side arrays, no fence.
template <bool LOSSY = false, bool PAIR = false, class A>
__device__ __forceinline__ void publish_any(TileStatus st, uint64_t t, uint64_t state, A v) {
    if constexpr (PAIR) {
        static_assert(sizeof(A) == 8, "word pairs carry 8-byte values");
        const uint64_t b = to_bits(v);
        store<Order::Release, Scope::Device>(&st.words[2 * t], (uint64_t)((b & 0xFFFFFFFF00000000ull) | state));
        store<Order::Release, Scope::Device>(&st.words[2 * t + 1], (uint64_t)((b << 32) | state));
        return;
    }
    uint64_t packed;
    if (pack_value<LOSSY>(v, packed)) {
        store<Order::Release, Scope::Device>(&st.words[t], packed | state);
    } else {
        uint64_t* side = reinterpret_cast<uint64_t*>(state == kFlagPrefix ? st.incls : st.aggs);
        side[t] = to_bits(v);
        store<Order::Release, Scope::Device>(&st.words[t], kFlagWide | state);
    }
}

// head: tile t starts a segment (tile 0, or the first tile of a row in a segmented scan); its
// inclusive prefix is op(init, agg) at once, and no lookback passes it.
template <bool LOSSY = false, bool PAIR = false, class A, class F>
__device__ __forceinline__ void publish_aggregate_any(TileStatus st, uint64_t t, A agg, A init, F op, bool head) {
    if (head) publish_any<LOSSY, PAIR>(st, t, kFlagPrefix, op(init, agg));
    else publish_any<LOSSY, PAIR>(st, t, kFlagAgg, agg);
}
template <bool LOSSY = false, bool PAIR = false, class A, class F>
__device__ __forceinline__ void publish_aggregate_any(TileStatus st, uint64_t t, A agg, A init, F op) {
    publish_aggregate_any<LOSSY, PAIR>(st, t, agg, init, op, t == 0);
}

// Run by all 32 lanes of one warp after publish_aggregate_any(t).  Returns the exclusive prefix of
// tile t (init for a head tile) and publishes tile t's inclusive prefix.  The walk stops at the
// nearest inclusive prefix, so it never crosses a head tile into an earlier segment.
template <int K, bool LOSSY = false, bool PAIR = false, class A, class F>
__device__ __forceinline__ A decoupled_lookback_any(TileStatus st, uint64_t t, A agg, A init, A identity, F op,
                                                    uint32_t* status, uint64_t timeout_ns, bool head) {
    const unsigned lane = lane0();
    if (head) return init;
    A excl = identity;
    long long end = (long long)t - 1;
    uint64_t t_start = 0;
    bool timed_out = false;
    unsigned backoff = KI_LOOKBACK_MIN_SLEEP_NS;
    const uint64_t* aggs = reinterpret_cast<const uint64_t*>(st.aggs);
    const uint64_t* incls = reinterpret_cast<const uint64_t*>(st.incls);
    while (true) {
        uint64_t w[K], lo[K];
        int first_p, first_zero;
        int pos_p, pos_zero;
        while (true) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const long long idx = end - (long long)(lane * K + k);
                if constexpr (PAIR) {
                    w[k] = kFlagPrefix;
                    lo[k] = 0;
                    if (idx >= 0) {
                        w[k] = load<Order::Relaxed, Scope::Device>(&st.words[2 * idx]);
                        lo[k] = load<Order::Relaxed, Scope::Device>(&st.words[2 * idx + 1]);
                        if ((w[k] & 3) != (lo[k] & 3)) w[k] = kFlagNone;  // between two publishes
                    }
                } else {
                    w[k] = (idx >= 0) ? load<Order::Relaxed, Scope::Device>(&st.words[idx]) : kFlagPrefix;
                }
            }
            first_p = K;
            first_zero = K;
#pragma unroll
            for (int k = K - 1; k >= 0; --k) {
                if ((w[k] & 3) == kFlagPrefix) first_p = k;
                if ((w[k] & 3) == kFlagNone) first_zero = k;
            }
            const unsigned pm = __ballot_sync(0xffffffffu, first_p < K);
            const unsigned zm = __ballot_sync(0xffffffffu, first_zero < K);
            const int lp = pm ? __ffs(pm) - 1 : 32, lz = zm ? __ffs(zm) - 1 : 32;
            pos_p = (lp < 32) ? lp * K + __shfl_sync(0xffffffffu, first_p, lp) : 32 * K;
            pos_zero = (lz < 32) ? lz * K + __shfl_sync(0xffffffffu, first_zero, lz) : 32 * K;
            if (pos_zero > pos_p || (pos_zero == 32 * K && pos_p == 32 * K)) break;
            const uint64_t now = globaltimer_ns();
            if (t_start == 0) t_start = now;
            timed_out = __shfl_sync(0xffffffffu, (int)(now - t_start > timeout_ns), 0) != 0;
            if (timed_out) break;
            __nanosleep(backoff);
            if (backoff < KI_LOOKBACK_MAX_SLEEP_NS) backoff <<= 1;
        }
        if (timed_out) {
            if (lane == 0) atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
            break;
        }
        // values of the words at positions <= pos_p (all of the window when it holds no P)
        bool any_wide = false;
        A v = identity;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int p = (int)lane * K + k;
            if (p <= pos_p && p < 32 * K && end - p >= 0) {
                if constexpr (PAIR) v = op(v, from_bits<A>((w[k] & 0xFFFFFFFF00000000ull) | (lo[k] >> 32)));
                else if (w[k] & kFlagWide) any_wide = true;
                else v = op(v, unpack_value<A, LOSSY>(w[k]));
            }
        }
        if (__any_sync(0xffffffffu, any_wide)) {
            fence<Scope::Device, Order::AcqRel>();
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int p = (int)lane * K + k;
                const long long idx = end - p;
                if (p <= pos_p && p < 32 * K && idx >= 0 && (w[k] & kFlagWide)) {
                    const uint64_t b = ((w[k] & 3) == kFlagPrefix) ? load<Order::Relaxed, Scope::Device>(&incls[idx])
                                                                   : load<Order::Relaxed, Scope::Device>(&aggs[idx]);
                    v = op(v, from_bits<A>(b));
                }
            }
        }
        excl = op(excl, warpfold(v, op));
        if (pos_p < 32 * K) break;
        end -= 32 * K;
    }
    if (lane == 0) publish_any<LOSSY, PAIR>(st, t, kFlagPrefix, op(excl, agg));
    return excl;
}
template <int K, bool LOSSY = false, bool PAIR = false, class A, class F>
__device__ __forceinline__ A decoupled_lookback_any(TileStatus st, uint64_t t, A agg, A init, A identity, F op,
                                                    uint32_t* status, uint64_t timeout_ns) {
    return decoupled_lookback_any<K, LOSSY, PAIR>(st, t, agg, init, identity, op, status, timeout_ns, t == 0);
}

// ---------------------------------------------------------------------------------------------
// mbarrier + 1-D bulk copies (cp.async.bulk, no tensor map, no multicast)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase; returns false (and latches KI_DEV_TIMEOUT) on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* status,
                                                  uint64_t timeout_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > timeout_ns) {
            atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
            return false;
        }
    }
    return true;
}

// global -> shared bulk copy completing on `bar` (dst, src 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// As bulk_g2s, but the lines it brings into L2 are marked evict-last: for tiles that are read a
// second time from L2 shortly after (createpolicy.fractional.L2::evict_last, fraction 1.0).
__device__ __forceinline__ void bulk_g2s_keep(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// As bulk_g2s with an L2 eviction-priority policy made by createpolicy (evict_normal / _first / _last).
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// L2 eviction-priority policies for the .L2::cache_hint forms (fraction 1.0: every access).
__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Asynchronous prefetch of [src, src + bytes) into L2 (src 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src_gmem, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes) : "memory");
}

// shared -> global bulk copy in the current bulk group.
__device__ __forceinline__ void bulk_s2g(void* dst_gmem, const void* src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem),
                 "r"(smem_addr(src_smem)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until all committed bulk stores have finished (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace ki
