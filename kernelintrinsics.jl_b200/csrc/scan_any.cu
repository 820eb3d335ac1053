// scan_any.cu -- device-wide inclusive or exclusive scan for any of Base's +, max, min over Int32,
// UInt32, Int64, UInt64, Float32 and Float64 (Base.cumsum / accumulate(op, x; init)).
//
// The pipeline of scan.cu (one persistent CTA per SM, 31 work warps + 1 look warp, tiles taken in
// ticket order, 1-D TMA bulk staging, decoupled lookback of tile k-1 while tile k is summed, second
// pass from L2), generalised over the element type T and the operator:
//   * a tile is 124 KiB of input: 15872 elements of 8 bytes or 31744 of 4 bytes; a row is 32 lanes x
//     one 16-byte vector (2 or 4 elements per lane), a warp owns 8 rows;
//   * values are accumulated in Traits<T, Op>::A (ki/ops.cuh: 64-bit integers for Int32/UInt32 sums,
//     Float64 for Float32 sums) and written as Traits<T, Op>::R (Int64/UInt64 for widened sums,
//     Float32 for Float32 sums, T otherwise), as Base.cumsum does;
//   * tile aggregates and prefixes ride in the status words when they fit (4-byte values, 8-byte
//     integers within 61 bits) and otherwise travel through the lookback's side arrays
//     (decoupled_lookback_any in ki/lookback.cuh).
// The Int64 + scan keeps its own kernel (scan.cu), whose values travel packed in the status words.
//
// Exclusive scans write op(init, x[1..i-1]) at i (init at the first element); inclusive scans
// op(init, x[1..i]).  Float sums are deterministic up to the order in which lookback windows find
// their predecessors, i.e. to Float64 rounding before the final Float32 rounding.
#include "ki/common.cuh"
#include "ki/intrinsics.cuh"
#include "ki/lookback.cuh"
#include "ki/ops.cuh"

#include <limits>

namespace {

constexpr int kWorkWarps = 31;
constexpr int kLookWarp = kWorkWarps;
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kThreads = kWorkThreads + 32;
constexpr int kRowsPerWarp = 8;
constexpr size_t kTileBytes = (size_t)kWorkWarps * kRowsPerWarp * 32 * 16;  // 126976 B

template <class T>
struct Shape {
    static constexpr int kE = (int)(16 / sizeof(T));        // elements per lane per row
    static constexpr int kRow = 32 * kE;                     // elements per row
    static constexpr int kSpan = kRowsPerWarp * kRow;         // elements per warp
    static constexpr int kTile = kWorkWarps * kSpan;          // elements per tile
};

struct AnyArgs {
    const void* in;
    void* out;
    size_t n;
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

template <class T, class Op>
__device__ __forceinline__ T pad_value() {  // the identity, as an input element
    if constexpr (std::is_same<Op, ki::JAdd>::value) return T(0);
    else if constexpr (std::is_same<Op, ki::JMax>::value) return ki::lowest_of<T>();
    else return ki::highest_of<T>();
}

template <class T, class Op, bool EXCL>
__global__ void __launch_bounds__(kThreads, 1) scan_any_kernel(AnyArgs a) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    using S = Shape<T>;
    constexpr int kE = S::kE;
    const ki::OpFn<T, Op> op;
    const A id = Tr::identity();
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
    const uint64_t ntiles = (a.n + S::kTile - 1) / S::kTile;
    auto bulk_ok = [&](uint64_t t) { return a.tma_in && t < ntiles && (t + 1) * (uint64_t)S::kTile <= a.n; };
    auto fetch = [&]() {
        const unsigned long long t = atomicAdd(a.ticket, 1ull);
        ticket = t;
        if (bulk_ok(t)) {
            ki::fence_proxy_async_smem();
            ki::mbar_arrive_expect_tx(&bar, (uint32_t)kTileBytes);
            ki::bulk_g2s_keep(sb, in + t * S::kTile, (uint32_t)kTileBytes, &bar);
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
                const A ex = ki::decoupled_lookback_any<1>(a.st, o.t, o.agg, init, id, op, a.status, a.timeout_ns);
                if (lane == 0) o.tile_excl = ex;
            }
        } else if (new_valid) {
            const size_t first = (size_t)t_new * S::kTile;
            const int count = (int)min((size_t)S::kTile, a.n - first);
            if (bulk_ok(t_new)) {
                if (!ki::mbar_wait_bounded(&bar, phase, a.status, a.timeout_ns))
                    ki::mbar_wait_bounded(&bar, phase, a.status, a.timeout_ns);  // never leave a copy in flight
                phase ^= 1u;
            } else {
                const T pad = pad_value<T, Op>();
                for (int i = tid; i < S::kTile; i += kWorkThreads) sb[i] = (i < count) ? in[first + i] : pad;
                work_sync();
            }
            A s = id;
#pragma unroll
            for (int j = 0; j < kRowsPerWarp; ++j) {
                const ki::Vec16<T> v = *reinterpret_cast<const ki::Vec16<T>*>(sb + w * S::kSpan + S::kRow * j + kE * lane);
#pragma unroll
                for (int e = 0; e < kE; ++e) s = op(s, Tr::lift(v.v[e]));
            }
            s = ki::warpfold(s, op);
            if (lane == 0) warp_tot[w] = s;
            work_sync();
            if (w == 0) {
                const A x = (lane < (unsigned)kWorkWarps) ? warp_tot[lane] : id;
                const A inc = ki::warpreduce(x, op);
                A exc = __shfl_up_sync(0xffffffffu, inc, 1);
                if (lane == 0) exc = id;
                const A agg = __shfl_sync(0xffffffffu, inc, kWorkWarps - 1);
                PendingAny<A>& e = slot[cur];
                if (lane < (unsigned)kWorkWarps) e.warp_excl[lane] = exc;
                if (lane == 0) {
                    e.t = t_new;
                    e.agg = agg;
                    ki::publish_aggregate_any(a.st, t_new, agg, init, op);
                }
            }
        }
        __syncthreads();

        // ---- phase B: start tile k+1's load; finish tile k-1 -----------------------------------------
        if (tid == kLookWarp * 32 && new_valid) fetch();
        if (w < kWorkWarps && have_old) {
            const PendingAny<A>& o = slot[cur ^ 1];
            const size_t first = (size_t)o.t * S::kTile;
            const int count = (int)min((size_t)S::kTile, a.n - first);
            const bool full = count == S::kTile;
            A carry = op(o.tile_excl, o.warp_excl[w]);
            ki::Vec16<T> v[kRowsPerWarp];
            const T pad = pad_value<T, Op>();
#pragma unroll
            for (int j = 0; j < kRowsPerWarp; ++j) {
                const int i = w * S::kSpan + S::kRow * j + kE * (int)lane;
                if (full && a.tma_in) {
                    const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(in + first + i));
                    v[j] = *reinterpret_cast<const ki::Vec16<T>*>(&raw);
                } else {
#pragma unroll
                    for (int e = 0; e < kE; ++e) v[j].v[e] = (i + e < count) ? in[first + i + e] : pad;
                }
            }
#pragma unroll
            for (int j = 0; j < kRowsPerWarp; ++j) {
                A part[kE];  // inclusive prefixes of this lane's elements
                part[0] = Tr::lift(v[j].v[0]);
#pragma unroll
                for (int e = 1; e < kE; ++e) part[e] = op(part[e - 1], Tr::lift(v[j].v[e]));
                const A inc = ki::warpreduce(part[kE - 1], op);
                A before = __shfl_up_sync(0xffffffffu, inc, 1);
                if (lane == 0) before = id;
                const A base = op(carry, before);
                alignas(16) R r[kE];
#pragma unroll
                for (int e = 0; e < kE; ++e) {
                    if (EXCL) r[e] = Tr::lower(e == 0 ? base : op(base, part[e - 1]));
                    else r[e] = Tr::lower(op(base, part[e]));
                }
                const int i = w * S::kSpan + S::kRow * j + kE * (int)lane;
                if (full && a.vec_out) {
                    constexpr int kStores = (int)(kE * sizeof(R) / 16);
#pragma unroll
                    for (int q = 0; q < kStores; ++q)
                        __stcs(reinterpret_cast<uint4*>(out + first + i) + q, reinterpret_cast<const uint4*>(r)[q]);
                } else {
#pragma unroll
                    for (int e = 0; e < kE; ++e)
                        if (i + e < count) out[first + i + e] = r[e];
                }
                carry = op(carry, __shfl_sync(0xffffffffu, inc, 31));
            }
        }
        __syncthreads();
        have_old = new_valid;
        cur ^= 1;
    }
}

template <class T, class Op>
int scan_launch(ki_ctx* ctx, bool excl, const void* d_in, void* d_out, size_t n, const void* h_init, cudaStream_t s) {
    using Tr = ki::Traits<T, Op>;
    using A = typename Tr::A;
    using R = typename Tr::R;
    using S = Shape<T>;
    if (!ki::aligned(d_in, sizeof(T)) || !ki::aligned(d_out, sizeof(R)))
        return ki::set_error(ctx, KI_ERR_ARG, "scan: misaligned input or output");
    const uintptr_t i0 = (uintptr_t)d_in, o0 = (uintptr_t)d_out;
    const uintptr_t ib = n * sizeof(T), ob = n * sizeof(R);
    if (!(i0 == o0 && sizeof(T) == sizeof(R)) && i0 < o0 + ob && o0 < i0 + ib)
        return ki::set_error(ctx, KI_ERR_ARG, "scan: input and output overlap (only an exact in-place scan is allowed)");
    // init: a host value of the result type, converted to the accumulation type; else the identity
    A init;
    if (h_init) {
        R r;
        memcpy(&r, h_init, sizeof(R));
        if constexpr (std::is_same<Op, ki::JAdd>::value) init = (A)r;
        else init = Tr::lift(r);
    } else if constexpr (std::is_same<Op, ki::JAdd>::value) {
        init = A(0);
    } else {
        using TT = typename std::conditional<std::is_floating_point<T>::value, T, double>::type;
        if constexpr (std::is_floating_point<T>::value)
            init = Tr::lift(std::is_same<Op, ki::JMax>::value ? -std::numeric_limits<TT>::infinity()
                                                               : std::numeric_limits<TT>::infinity());
        else
            init = std::is_same<Op, ki::JMax>::value ? std::numeric_limits<A>::lowest() : std::numeric_limits<A>::max();
    }
    const size_t ntiles = (n + S::kTile - 1) / S::kTile;
    const size_t words_off = 256;
    void* base = nullptr;
    int rc = ki::ensure_region(ctx, KI_REG_SCAN_ANY, words_off + ntiles * 24, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    KI_CUDA(ctx, cudaMemsetAsync(b, 0, words_off + ntiles * sizeof(uint64_t), s));
    AnyArgs a;
    a.in = d_in;
    a.out = d_out;
    a.n = n;
    a.init_bits = 0;
    memcpy(&a.init_bits, &init, sizeof(A));
    a.st.words = reinterpret_cast<uint64_t*>(b + words_off);
    a.st.aggs = reinterpret_cast<int64_t*>(b + words_off + ntiles * 8);
    a.st.incls = reinterpret_cast<int64_t*>(b + words_off + ntiles * 16);
    a.ticket = reinterpret_cast<unsigned long long*>(b);
    a.status = ctx->d_status;
    a.timeout_ns = ctx->wait_timeout_ns;
    a.tma_in = ki::aligned(d_in, 16);
    a.vec_out = ki::aligned(d_out, 16);
    size_t grid = (size_t)ctx->sm_count;
    if (grid > ntiles) grid = ntiles;
    if (excl) {
        KI_CUDA(ctx, cudaFuncSetAttribute(scan_any_kernel<T, Op, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kTileBytes));
        scan_any_kernel<T, Op, true><<<(unsigned)grid, kThreads, kTileBytes, s>>>(a);
    } else {
        KI_CUDA(ctx, cudaFuncSetAttribute(scan_any_kernel<T, Op, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kTileBytes));
        scan_any_kernel<T, Op, false><<<(unsigned)grid, kThreads, kTileBytes, s>>>(a);
    }
    return ki::check_launch(ctx, "scan_any_kernel launch");
}

template <class Op>
int scan_dtype(ki_ctx* ctx, int dtype, bool excl, const void* d_in, void* d_out, size_t n, const void* h_init,
               cudaStream_t s) {
    switch (dtype) {
        case KI_I32: return scan_launch<int32_t, Op>(ctx, excl, d_in, d_out, n, h_init, s);
        case KI_U32: return scan_launch<uint32_t, Op>(ctx, excl, d_in, d_out, n, h_init, s);
        case KI_I64: return scan_launch<int64_t, Op>(ctx, excl, d_in, d_out, n, h_init, s);
        case KI_U64: return scan_launch<uint64_t, Op>(ctx, excl, d_in, d_out, n, h_init, s);
        case KI_F32: return scan_launch<float, Op>(ctx, excl, d_in, d_out, n, h_init, s);
        case KI_F64: return scan_launch<double, Op>(ctx, excl, d_in, d_out, n, h_init, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "scan: dtype must be Int32/UInt32/Int64/UInt64/Float32/Float64");
    }
}

}  // namespace

extern "C" int ki_scan(ki_ctx* ctx, int op, int dtype, int exclusive, const void* d_in, void* d_out, size_t n,
                       const void* h_init, void* stream) {
    KI_CHECK_CTX(ctx);
    if (n == 0) return KI_OK;
    if (!d_in || !d_out) return ki::set_error(ctx, KI_ERR_ARG, "scan: null pointer");
    KI_GUARD(ctx);
    cudaStream_t s = ki::as_stream(stream);
    const bool excl = exclusive != 0;
    switch (op) {
        case KI_OP_ADD: return scan_dtype<ki::JAdd>(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_MAX: return scan_dtype<ki::JMax>(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        case KI_OP_MIN: return scan_dtype<ki::JMin>(ctx, dtype, excl, d_in, d_out, n, h_init, s);
        default: return ki::set_error(ctx, KI_ERR_ARG, "scan: op must be KI_OP_ADD, KI_OP_MAX or KI_OP_MIN");
    }
}
