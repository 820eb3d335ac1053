// ki/lookback.cuh -- decoupled lookback over per-tile status words, and 1-D TMA bulk helpers.
//
// Tile status (one entry per tile, reset to 0 before each call):
//   flags[t] : 0 = nothing published, 1 = aggregate published (A), 2 = inclusive prefix (P)
//   aggs[t]  : the tile's own aggregate          (valid once flags[t] >= 1)
//   incls[t] : inclusive prefix through tile t    (valid once flags[t] == 2)
// A value is written with a plain store, then the flag with st.release.gpu; readers load the flag
// with ld.acquire.gpu and then the value with ld.relaxed.gpu.  These are the @access store /
// load defaults of the reference (src/macros.jl:259-275 -> ext/CUDA/scopes_ordering.jl:89-193).
//
// Every wait is bounded by %globaltimer: when it runs out the warp latches KI_DEV_TIMEOUT in the
// context's status word and carries on with what it has, so the grid always finishes.
#pragma once

#include <cstdint>

#include "common.cuh"
#include "intrinsics.cuh"

namespace ki {

constexpr uint64_t kFlagNone = 0, kFlagAgg = 1, kFlagPrefix = 2;

struct TileStatus {
    uint64_t* flags;
    int64_t* aggs;
    int64_t* incls;
};

// Run by all 32 lanes of one warp.  Publishes tile t's aggregate, looks back over predecessors
// until an inclusive prefix is found, publishes tile t's inclusive prefix and returns the exclusive
// prefix of tile t (including `seed`).  Sums wrap around (two's complement).
__device__ __forceinline__ int64_t decoupled_lookback(TileStatus st, uint64_t t, int64_t agg, int64_t seed,
                                                      uint32_t* status, uint64_t timeout_ns) {
    const unsigned lane = lane0();
    if (t == 0) {
        if (lane == 0) {
            st.incls[0] = wrap_add(seed, agg);
            store<Order::Release, Scope::Device>(&st.flags[0], kFlagPrefix);
        }
        return seed;
    }
    if (lane == 0) {
        st.aggs[t] = agg;
        store<Order::Release, Scope::Device>(&st.flags[t], kFlagAgg);
    }
    int64_t excl = 0;
    long long end = (long long)t - 1;  // window = tiles end-31 .. end, lane k looks at end-k
    uint64_t t_start = 0;
    bool timed_out = false;
    while (true) {
        const long long idx = end - (long long)lane;
        uint64_t f;
        unsigned pending;
        while (true) {
            f = (idx >= 0) ? load<Order::Acquire, Scope::Device>(&st.flags[idx]) : kFlagPrefix;
            pending = __ballot_sync(0xffffffffu, f == kFlagNone);
            if (!pending) break;
            const uint64_t now = globaltimer_ns();
            if (t_start == 0) t_start = now;
            timed_out = __shfl_sync(0xffffffffu, (int)(now - t_start > timeout_ns), 0) != 0;
            if (timed_out) break;
            __nanosleep(32);
        }
        if (timed_out) {
            if (lane == 0) atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
            break;
        }
        int64_t v = 0;
        if (idx >= 0) {
            if (f == kFlagPrefix) v = load<Order::Relaxed, Scope::Device>(&st.incls[idx]);
            else v = load<Order::Relaxed, Scope::Device>(&st.aggs[idx]);
        }
        const unsigned pmask = __ballot_sync(0xffffffffu, f == kFlagPrefix);
        if (pmask) {
            const unsigned first = (unsigned)(__ffs(pmask) - 1);
            if (lane > first) v = 0;
            excl = wrap_add(excl, warpfold(v, WrapAdd{}));
            break;
        }
        excl = wrap_add(excl, warpfold(v, WrapAdd{}));
        end -= 32;
    }
    if (lane == 0) {
        st.incls[t] = wrap_add(excl, agg);
        store<Order::Release, Scope::Device>(&st.flags[t], kFlagPrefix);
    }
    return excl;
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
