// gemm_e4m3.cu -- fp8 e4m3 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// C (M x N, Float32, row-major) = alpha * A (M x K, e4m3, row-major) * B (K x N, e4m3, row-major)
//
// Two persistent kernels.  gemm_e4m3_pair_kernel (further down) runs when M and N are multiples of
// 256: clusters of two CTAs share 256 x 256 tiles through tcgen05.mma.cta_group::2.  Otherwise
// gemm_e4m3_kernel, one CTA of 6 warps per SM, 128 x 256 output tiles, K blocks of 128:
//   warp 0     TMA producer: 2-D tiled bulk-tensor loads (128B swizzle) of A (128 x 128 B, K-major)
//              and B (2 x 128 K-rows x 128 B, N-major) into a 4-stage shared-memory ring;
//   warp 1     allocates 512 TMEM columns (two 128 x 256 Float32 accumulators) and issues
//              tcgen05.mma.cta_group::1.kind::f8f6f4 (M=128, N=256, K=32) from one thread;
//              tcgen05.commit releases ring stages and hands finished accumulators on;
//   warps 2-5  epilogue: tcgen05.ld 32x32b.x32 from the warp's TMEM lane quadrant, scale by alpha,
//              stage 32 x 32 Float32 blocks in swizzled shared memory, TMA-store them.
// The double-buffered accumulator lets the epilogue of tile i overlap the main loop of tile i+1.
// No cluster multicast anywhere: every CTA loads its own tiles.
//
// Shared-memory descriptors (tcgen05 matrix descriptor): start address >> 4 in bits 0-13,
// leading-dimension byte offset >> 4 in bits 16-29, stride-dimension byte offset >> 4 in bits
// 32-45, descriptor version 1 in bits 46-47, layout type in bits 61-63 (2 = 128-byte swizzle).
//   A, K-major:  rows of 128 B (one swizzle row), 8-row groups 1024 B apart (SBO); LBO unused (1).
//                The k-th K=32 slice starts 32 B further.
//   B, N-major:  each 128-element N block is 128 K-rows x 128 B; 8-row K groups 1024 B apart (SBO),
//                N blocks 16 KiB apart (LBO).  The k-th K=32 slice starts 32 rows (4 KiB) further.
// Instruction descriptor (kind::f8f6f4): D format F32 (bits 4-5 = 1), A and B e4m3 (0), A K-major
// (bit 15 = 0), B MN-major (bit 16 = 1), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
//
// Every mbarrier wait is bounded by %globaltimer; a role that gives up latches KI_DEV_TIMEOUT,
// raises the CTA abort flag and the others leave their loops at their next wait.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"

#ifndef KI_GEMM_PAIRS
#define KI_GEMM_PAIRS 1  // use the CTA-pair kernel where M and N are multiples of 256
#endif

namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4, ACCS = 2;
constexpr int A_BYTES = BM * BK;               // 16 KiB
constexpr int B_HALF_BYTES = BK * 128;         // 16 KiB per 128-wide N block
constexpr int B_BYTES = 2 * B_HALF_BYTES;      // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES; // 48 KiB
constexpr int EPI_COLS = 32;
constexpr int EPI_BUF_BYTES = 32 * EPI_COLS * 4;  // 32 rows x 32 Float32 = 4 KiB
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr int TMEM_COLS = ACCS * BN;           // 512
constexpr int RING_BYTES = STAGES * STAGE_BYTES;
constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_BUF_BYTES;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;

constexpr uint32_t IDESC = (1u << 4)            // D = F32
                           | (0u << 7) | (0u << 10)  // A, B = e4m3
                           | (0u << 15)         // A K-major
                           | (1u << 16)         // B MN-major
                           | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ uint64_t make_desc(uint32_t smem, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((smem >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

#ifndef KI_GEMM_C_EVICT_FIRST
#define KI_GEMM_C_EVICT_FIRST 1
#endif
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, uint32_t src) {
#if KI_GEMM_C_EVICT_FIRST
    // C is written once and not read again here: evict-first, so the A and B panels stay in L2
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::"l"(map),
        "r"(c0), "r"(c1), "r"(src), "l"(policy)
        : "memory");
#else
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
                 "r"(c1), "r"(src)
                 : "memory");
#endif
}

__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; on timeout (or when another role already aborted) returns false.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort, uint32_t* status,
                                         uint64_t timeout_ns) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = ki::globaltimer_ns();
    while (!mbar_try(bar, parity)) {
        if (*abort) return false;
        if (ki::globaltimer_ns() - t0 > timeout_ns) {
            *abort = 1;
            atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Bounded wait that ignores the abort flag: used to drain copies and MMAs still in flight.
__device__ __forceinline__ void wait_drain(uint32_t bar, uint32_t parity, uint32_t* status, uint64_t timeout_ns) {
    const uint64_t t0 = ki::globaltimer_ns();
    while (!mbar_try(bar, parity)) {
        if (ki::globaltimer_ns() - t0 > timeout_ns) {
            atomicOr(status, (uint32_t)KI_DEV_TIMEOUT);
            return;
        }
    }
}

#define KI_TMEM_LD_X32(taddr, v)                                                                           \
    asm volatile(                                                                                             \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17," \
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                    \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),       \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),  \
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),            \
          "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),            \
          "=r"(v[30]), "=r"(v[31])                                                                            \
        : "r"(taddr))

// Output tile t -> (m block, n block): groups of KI_GEMM_GROUP_M m blocks are walked n-block by
// n-block, so the tiles in flight at once share a few A row panels and B column panels that stay in
// L2.  At 8192^3 with CTA pairs: m fastest over the whole matrix 2469 TFLOP/s, groups of 4 / 8 / 16
// / 20 / 24 m blocks 2550 / 2633 / 2756 / 2708 / 2666, groups of 8 / 16 n blocks 2718 / 2724.
// With evict-first C stores (the A and B panels keep more of L2): groups of 16 / 24 / 32 m blocks
// 2847 / 2778 / 2654 on one box, and 2765 -> 2780-2794 against plain C stores on another.
// Evict-last hints on the A or the B tile loads as well: 2702 / 2682 against 2708-2750 without.
#ifndef KI_GEMM_GROUP_M
#define KI_GEMM_GROUP_M 16  // 0: one group of all m blocks; negative: groups of n blocks
#endif
__device__ __forceinline__ void group_coords(int t, int g, int num_a, int num_b, int& a, int& b) {
    const int grp = t / (g * num_b);
    const int first = grp * g;
    const int gsz = min(g, num_a - first);
    const int in = t - grp * g * num_b;
    a = first + in % gsz;
    b = in / gsz;
}
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
    if (KI_GEMM_GROUP_M >= 0) group_coords(t, KI_GEMM_GROUP_M > 0 ? KI_GEMM_GROUP_M : num_m, num_m, num_n, mb, nb);
    else group_coords(t, -KI_GEMM_GROUP_M, num_n, num_m, nb, mb);  // groups of n blocks instead
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_e4m3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, int M, int N, int K, float alpha, uint32_t* status,
                     uint64_t timeout_ns) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = ki::smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-aligned: 128B-swizzle atoms
    const uint32_t ring = base;
    const uint32_t epi = base + RING_BYTES;
    const uint32_t bars = epi + EPI_BYTES;
    const uint32_t full0 = bars, empty0 = bars + 8 * STAGES, tfull0 = bars + 16 * STAGES;
    const uint32_t tempty0 = tfull0 + 8 * ACCS;
    const uint32_t drain = tempty0 + 8 * ACCS;
    uint8_t* gbase = smem_raw + (base - raw);
    const int misc = RING_BYTES + EPI_BYTES + 16 * STAGES + 16 * ACCS + 8;
    volatile int* abort = reinterpret_cast<volatile int*>(gbase + misc);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gbase + misc + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * s));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(empty0 + 8 * s));
        }
        for (int b = 0; b < ACCS; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tfull0 + 8 * b));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tempty0 + 8 * b), "r"(EPI_WARPS));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(drain));
        *abort = 0;
        ki::fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmC) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         ki::smem_addr(tmem_holder)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    const int num_m = M / BM, num_n = N / BN, tiles = num_m * num_n, kblocks = K / BK;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 1;  // a fresh barrier's preceding phase counts as complete
            uint32_t issued_ph[STAGES];
            bool issued[STAGES];
            for (int k = 0; k < STAGES; ++k) issued[k] = false;
            for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
                int mb, nb;
                tile_coords(tile, num_m, num_n, mb, nb);
                const int m0 = mb * BM, n0 = nb * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!wait_bar(empty0 + 8 * s, ph, abort, status, timeout_ns)) break;
                    const uint32_t sa = ring + s * STAGE_BYTES, sb = sa + A_BYTES;
                    mbar_expect_tx(full0 + 8 * s, STAGE_BYTES);
                    tma_load_2d(sa, &tmA, kb * BK, m0, full0 + 8 * s);
                    tma_load_2d(sb, &tmB, n0, kb * BK, full0 + 8 * s);
                    tma_load_2d(sb + B_HALF_BYTES, &tmB, n0 + 128, kb * BK, full0 + 8 * s);
                    issued[s] = true;
                    issued_ph[s] = ph ^ 1;  // the full-barrier phase this issue completes
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            // After an abort, loads may still be in flight: wait (bounded) until each landed
            // before the shared memory they target is released.
            if (*abort) {
                for (int k = 0; k < STAGES; ++k)
                    if (issued[k]) wait_drain(full0 + 8 * k, issued_ph[k], status, timeout_ns);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0, acc = 0;
            uint32_t ph_full = 0, ph_empty = 1;
            for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
                if (!wait_bar(tempty0 + 8 * acc, ph_empty, abort, status, timeout_ns)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * BN);
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!wait_bar(full0 + 8 * s, ph_full, abort, status, timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = ring + s * STAGE_BYTES, sb = sa + A_BYTES;
                    const uint64_t adesc = make_desc(sa, 16, 1024);
                    const uint64_t bdesc = make_desc(sb, B_HALF_BYTES, 1024);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_f8(d, adesc + (uint64_t)((k * 32) >> 4), bdesc + (uint64_t)((k * 32 * 128) >> 4),
                               (kb | k) != 0);
                    mma_commit(empty0 + 8 * s);
                    if (++s == STAGES) {
                        s = 0;
                        ph_full ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * acc);
                if (++acc == ACCS) {
                    acc = 0;
                    ph_empty ^= 1;
                }
            }
            // Every MMA this thread issued has finished before TMEM and the ring are released.
            mma_commit(drain);
            wait_drain(drain, 0, status, timeout_ns);
        }
    } else {
        const int ew = warp - 2;          // epilogue warp 0..3
        const int q = warp & 3;           // TMEM lane quadrant this warp may access
        const int row0 = q * 32;
        int acc = 0, buf = 0;
        uint32_t ph = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            int mb, nb;
            tile_coords(tile, num_m, num_n, mb, nb);
            const int m0 = mb * BM, n0 = nb * BN;
            int ok = 0;
            if (lane == 0) ok = wait_bar(tfull0 + 8 * acc, ph, abort, status, timeout_ns) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);  // one decision for the whole warp
            if (!ok) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < BN / EPI_COLS; ++c) {
                uint32_t v[32];
                const uint32_t taddr = tmem + ((uint32_t)row0 << 16) + (uint32_t)(acc * BN + c * EPI_COLS);
                KI_TMEM_LD_X32(taddr, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (c == BN / EPI_COLS - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
                }
                if (lane == 0) bulk_wait_read_le1();
                __syncwarp();
                const uint32_t sbuf = epi + (uint32_t)((ew * 2 + buf) * EPI_BUF_BYTES);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t addr = sbuf + (uint32_t)lane * 128u + (uint32_t)(((j ^ (lane & 7)) << 4));
                    const float f0 = __uint_as_float(v[4 * j + 0]) * alpha, f1 = __uint_as_float(v[4 * j + 1]) * alpha;
                    const float f2 = __uint_as_float(v[4 * j + 2]) * alpha, f3 = __uint_as_float(v[4 * j + 3]) * alpha;
                    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(f0), "f"(f1), "f"(f2),
                                 "f"(f3)
                                 : "memory");
                }
                ki::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmC, n0 + c * EPI_COLS, m0 + row0, sbuf);
                    ki::bulk_commit();
                }
                buf ^= 1;
            }
            if (++acc == ACCS) {
                acc = 0;
                ph ^= 1;
            }
        }
        if (lane == 0) ki::bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// CTA-pair variant: cluster of 2 CTAs on 2 SMs, 256 x 256 output tiles, tcgen05.mma.cta_group::2.
//
// CTA rank r of the pair loads A rows [m0 + 128 r, +128) and B columns [n0 + 128 r, +128) of each
// K block into its own shared memory (no multicast: every CTA loads only its own half).  Both CTAs'
// loads complete on the full barrier of rank 0 (.cta_group::2 lets the peer's copy signal it), and
// rank 0's MMA thread issues M=256 N=256 K=32 MMAs that read A and B from both CTAs' shared memory
// at the same offsets; each CTA's TMEM receives its 128 rows x 256 columns.  Per SM this moves
// 32 KiB per K block for a 128 x 256 x 128 product instead of 48 KiB, so six stages fit beside the
// epilogue staging and the shared-memory ingress per flop falls by a third.  (Storing the epilogue
// straight from registers to free a seventh stage was slower: 2472 against 2633 TFLOP/s.)  The MMA thread's commits arrive on the empty /
// accumulator-full barriers of both CTAs (one commit per CTA); the epilogue warps of both CTAs
// arrive on rank 0's accumulator-empty barrier.
// ---------------------------------------------------------------------------------------------
constexpr int STAGES2 = 6;
constexpr int STAGE2_BYTES = A_BYTES + B_HALF_BYTES;  // 32 KiB per CTA
constexpr int RING2_BYTES = STAGES2 * STAGE2_BYTES;
constexpr int SMEM2_BYTES = 1024 + RING2_BYTES + EPI_BYTES + BAR_BYTES;
constexpr uint32_t IDESC2 = (1u << 4)             // D = F32
                            | (0u << 7) | (0u << 10)  // A, B = e4m3
                            | (0u << 15)          // A K-major
                            | (1u << 16)          // B MN-major
                            | ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tile load into this CTA's shared memory whose completion is counted on `bar_cluster`, a barrier
// of either CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(dst),
        "l"(map), "r"(c0), "r"(c1), "r"(bar_cluster)
        : "memory");
}

__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC2), "r"(accumulate)
        : "memory");
}

// Arrive (once) on a barrier of either CTA when all earlier pair MMAs of this thread are done.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_e4m3_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, int M, int N, int K, float alpha,
                          uint32_t* status, uint64_t timeout_ns) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = ki::smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // identical in both CTAs: same kernel, same layout
    const uint32_t ring = base;
    const uint32_t epi = base + RING2_BYTES;
    const uint32_t bars = epi + EPI_BYTES;
    const uint32_t full0 = bars, empty0 = bars + 8 * STAGES2, tfull0 = bars + 16 * STAGES2;
    const uint32_t tempty0 = tfull0 + 8 * ACCS;
    const uint32_t drain = tempty0 + 8 * ACCS;
    uint8_t* gbase = smem_raw + (base - raw);
    const int misc = RING2_BYTES + EPI_BYTES + 16 * STAGES2 + 16 * ACCS + 8;
    volatile int* abort = reinterpret_cast<volatile int*>(gbase + misc);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gbase + misc + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES2; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * s));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(empty0 + 8 * s));
        }
        for (int b = 0; b < ACCS; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tfull0 + 8 * b));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tempty0 + 8 * b), "r"(2 * EPI_WARPS));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(drain));
        *abort = 0;
        ki::fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmC) : "memory");
    }
    if (warp == 1) {  // the same warp in both CTAs allocates the pair's TMEM together
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         ki::smem_addr(tmem_holder)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers are initialised before any copy or arrive crosses over
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    const int num_m = M / 256, num_n = N / 256, tiles = num_m * num_n, kblocks = K / BK;
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full_lead0 = map_rank(full0, 0);
            int s = 0;
            uint32_t ph = 1;  // a fresh barrier's preceding phase counts as complete
            uint32_t issued_ph[STAGES2];
            bool issued[STAGES2];
            for (int k = 0; k < STAGES2; ++k) issued[k] = false;
            for (int tile = pair; tile < tiles && !*abort; tile += pairs) {
                int mb, nb;
                tile_coords(tile, num_m, num_n, mb, nb);
                const int m0 = mb * 256 + 128 * (int)rank, n0 = nb * 256 + 128 * (int)rank;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!wait_bar(empty0 + 8 * s, ph, abort, status, timeout_ns)) break;
                    const uint32_t sa = ring + s * STAGE2_BYTES, sb = sa + A_BYTES;
                    if (leader) mbar_expect_tx(full0 + 8 * s, 2 * STAGE2_BYTES);  // both CTAs' bytes
                    tma_load_2d_pair(sa, &tmA, kb * BK, m0, full_lead0 + 8 * s);
                    tma_load_2d_pair(sb, &tmB, n0, kb * BK, full_lead0 + 8 * s);
                    issued[s] = true;
                    issued_ph[s] = ph ^ 1;
                    if (++s == STAGES2) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            if (*abort) {
                if (leader) {  // loads may still be in flight into both CTAs: wait (bounded) for them
                    for (int k = 0; k < STAGES2; ++k)
                        if (issued[k]) wait_drain(full0 + 8 * k, issued_ph[k], status, timeout_ns);
                } else {  // this CTA cannot observe rank 0's barrier: give its last loads time to land
                    const uint64_t t0 = ki::globaltimer_ns();
                    while (ki::globaltimer_ns() - t0 < 200000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            const uint32_t empty_peer0 = map_rank(empty0, 1), tfull_peer0 = map_rank(tfull0, 1);
            int s = 0, acc = 0;
            uint32_t ph_full = 0, ph_empty = 1;
            for (int tile = pair; tile < tiles && !*abort; tile += pairs) {
                if (!wait_bar(tempty0 + 8 * acc, ph_empty, abort, status, timeout_ns)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * BN);
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!wait_bar(full0 + 8 * s, ph_full, abort, status, timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = ring + s * STAGE2_BYTES, sb = sa + A_BYTES;
                    const uint64_t adesc = make_desc(sa, 16, 1024);
                    const uint64_t bdesc = make_desc(sb, B_HALF_BYTES, 1024);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_f8_pair(d, adesc + (uint64_t)((k * 32) >> 4), bdesc + (uint64_t)((k * 32 * 128) >> 4),
                                    (kb | k) != 0);
                    mma_commit_pair(empty0 + 8 * s);       // this CTA's stage is free again
                    mma_commit_pair(empty_peer0 + 8 * s);  // and the peer's
                    if (++s == STAGES2) {
                        s = 0;
                        ph_full ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit_pair(tfull0 + 8 * acc);
                mma_commit_pair(tfull_peer0 + 8 * acc);
                if (++acc == ACCS) {
                    acc = 0;
                    ph_empty ^= 1;
                }
            }
            mma_commit_pair(drain);  // every MMA issued has finished before TMEM and the rings go
            wait_drain(drain, 0, status, timeout_ns);
        }
    } else {
        const int ew = warp - 2;  // epilogue warp 0..3
        const int q = warp & 3;   // TMEM lane quadrant this warp may access
        const int row0 = q * 32;
        const uint32_t tempty_lead0 = map_rank(tempty0, 0);
        int acc = 0, buf = 0;
        uint32_t ph = 0;
        for (int tile = pair; tile < tiles; tile += pairs) {
            int mb, nb;
            tile_coords(tile, num_m, num_n, mb, nb);
            const int m0 = mb * 256 + 128 * (int)rank, n0 = nb * 256;
            int ok = 0;
            if (lane == 0) ok = wait_bar(tfull0 + 8 * acc, ph, abort, status, timeout_ns) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < BN / EPI_COLS; ++c) {
                uint32_t v[32];
                const uint32_t taddr = tmem + ((uint32_t)row0 << 16) + (uint32_t)(acc * BN + c * EPI_COLS);
                KI_TMEM_LD_X32(taddr, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (c == BN / EPI_COLS - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(tempty_lead0 + 8 * acc);
                }
                if (lane == 0) bulk_wait_read_le1();
                __syncwarp();
                const uint32_t sbuf = epi + (uint32_t)((ew * 2 + buf) * EPI_BUF_BYTES);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t addr = sbuf + (uint32_t)lane * 128u + (uint32_t)(((j ^ (lane & 7)) << 4));
                    const float f0 = __uint_as_float(v[4 * j + 0]) * alpha, f1 = __uint_as_float(v[4 * j + 1]) * alpha;
                    const float f2 = __uint_as_float(v[4 * j + 2]) * alpha, f3 = __uint_as_float(v[4 * j + 3]) * alpha;
                    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(f0), "f"(f1), "f"(f2),
                                 "f"(f3)
                                 : "memory");
                }
                ki::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmC, n0 + c * EPI_COLS, m0 + row0, sbuf);
                    ki::bulk_commit();
                }
                buf ^= 1;
            }
            if (++acc == ACCS) {
                acc = 0;
                ph ^= 1;
            }
        }
        if (lane == 0) ki::bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // neither CTA leaves while the other may still read its shared memory or TMEM
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool encode_2d(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, CUtensorMapDataType dt, const void* ptr,
               uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapL2promotion promo) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int ki_gemm_e4m3_f32(ki_ctx* ctx, const uint8_t* d_A, const uint8_t* d_B, float* d_C, int M, int N, int K,
                                float scale_a, float scale_b, void* stream) {
    KI_CHECK_CTX(ctx);
    if (!d_A || !d_B || !d_C) return ki::set_error(ctx, KI_ERR_ARG, "gemm: null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || M % BM || N % BN || K % BK)
        return ki::set_error(ctx, KI_ERR_ARG, "gemm: need M %% %d == 0, N %% %d == 0, K %% %d == 0 (got %d %d %d)", BM,
                             BN, BK, M, N, K);
    if (!ki::aligned(d_A, 16) || !ki::aligned(d_B, 16) || !ki::aligned(d_C, 16))
        return ki::set_error(ctx, KI_ERR_ARG, "gemm: pointers must be 16-byte aligned");
    KI_GUARD(ctx);
    auto enc = get_encode();
    if (!enc) return ki::set_error(ctx, KI_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tA, tB, tC;
    if (!encode_2d(enc, &tA, CU_TENSOR_MAP_DATA_TYPE_UINT8, d_A, (uint64_t)K, (uint64_t)M, (uint64_t)K, BK, BM,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B) ||
        !encode_2d(enc, &tB, CU_TENSOR_MAP_DATA_TYPE_UINT8, d_B, (uint64_t)N, (uint64_t)K, (uint64_t)N, 128, BK,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B) ||
        !encode_2d(enc, &tC, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, d_C, (uint64_t)N, (uint64_t)M, (uint64_t)N * 4, EPI_COLS,
                   32, CU_TENSOR_MAP_L2_PROMOTION_NONE))
        return ki::set_error(ctx, KI_ERR_ARG, "gemm: tensor map encoding failed");
    cudaStream_t st = ki::as_stream(stream);
    const float alpha = scale_a * scale_b;
    if (M % 256 == 0 && N % 256 == 0 && KI_GEMM_PAIRS) {
        // CTA pairs: grid = as many pairs as can be resident at once (persistent), at most one per tile
        KI_CUDA(ctx, cudaFuncSetAttribute(gemm_e4m3_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          SMEM2_BYTES));
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = SMEM2_BYTES;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (ctx->gemm_pairs == 0) {
            int nc = 0;
            cfg.gridDim = dim3(2 * (ctx->sm_count / 2));
            if (cudaOccupancyMaxActiveClusters(&nc, gemm_e4m3_pair_kernel, &cfg) != cudaSuccess || nc < 1) {
                cudaGetLastError();
                nc = ctx->sm_count / 2;
            }
            ctx->gemm_pairs = nc;
        }
        const int tiles = (M / 256) * (N / 256);
        const int pairs = tiles < ctx->gemm_pairs ? tiles : ctx->gemm_pairs;
        cfg.gridDim = dim3(2 * pairs);
        KI_CUDA(ctx, cudaLaunchKernelEx(&cfg, gemm_e4m3_pair_kernel, tA, tB, tC, M, N, K, alpha, ctx->d_status,
                                        ctx->wait_timeout_ns));
        return ki::check_launch(ctx, "gemm_e4m3_pair_kernel launch");
    }
    KI_CUDA(ctx, cudaFuncSetAttribute(gemm_e4m3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    const int tiles = (M / BM) * (N / BN);
    const int grid = tiles < ctx->sm_count ? tiles : ctx->sm_count;
    gemm_e4m3_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(tA, tB, tC, M, N, K, alpha, ctx->d_status,
                                                        ctx->wait_timeout_ns);
    return ki::check_launch(ctx, "gemm_e4m3_kernel launch");
}
