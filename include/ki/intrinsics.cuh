// ki/intrinsics.cuh -- device intrinsics for sm_100a with KernelIntrinsics.jl semantics.
//
// Each group restates one reference intrinsic in CUDA C++ / hand-written PTX:
//   memory ordering  @fence / @access       src/macros.jl:198-282, src/scopes_orderings.jl:13-154,
//                                          ext/CUDA/scopes_ordering.jl:10-193
//   warp shuffles    @shfl                  src/warp.jl:16-64,114-192, ext/CUDA/shuffle_vote.jl:5-21
//   warp scan        @warpreduce            src/warp.jl:194-237
//   warp fold        @warpfold              src/warp.jl:239-282
//   warp vote        @vote                  src/warp.jl:66-106,284-351, ext/CUDA/shuffle_vote.jl:23-34
//   lane / warpsize  @laneid / @warpsize    src/macros.jl:103-128, ext/KernelIntrinsicsCUDAExt.jl:13-19
//   vector access    vload_multi / vstore_multi! / generate_partN
//                                          src/vectorization.jl:306-420, ext/CUDA/vectorization.jl:5-27
//
// Differences from the reference, all deliberate:
//   * argument validation that the reference does at macro-expansion time (ArgumentError) is a
//     static_assert here;
//   * warpfold() is an xor butterfly, so every lane holds the total (a superset of the reference
//     contract, where only lane 1 is guaranteed); warpfold_down() is the reference's exact Down form;
//   * @laneid is 1-based, as in the reference.
#pragma once

#include <cstdint>
#include <cstring>
#include <type_traits>

namespace ki {

constexpr int kWarpSize = 32;

// ---------------------------------------------------------------------------------------------
// Scope / ordering lattice (src/scopes_orderings.jl:13-120)
// ---------------------------------------------------------------------------------------------
enum class Scope { Default, Workgroup, Device, System };
enum class Order { Default, Weak, Volatile, Relaxed, Acquire, Release, AcqRel, SeqCst };

// PTX scope strings (ext/CUDA/scopes_ordering.jl:10-14): Workgroup->cta, Device->gpu, System->sys.
#define KI_SCOPE_STR_Workgroup "cta"
#define KI_SCOPE_STR_Device "gpu"
#define KI_SCOPE_STR_System "sys"

// fence: PTX has no acquire-only or release-only fence, so Acquire/Release/AcqRel all lower to
// fence.acq_rel.<scope> and SeqCst to fence.sc.<scope> (ext/CUDA/scopes_ordering.jl:16-46).
// Weak/Volatile/Relaxed are rejected, as @fence does (src/macros.jl:203-207).
template <Scope S = Scope::Device, Order O = Order::AcqRel>
__device__ __forceinline__ void fence() {
    static_assert(O == Order::Acquire || O == Order::Release || O == Order::AcqRel || O == Order::SeqCst ||
                      O == Order::Default,
                  "Fences allow synchronizing orderings only: Acquire, Release, AcqRel, or SeqCst.");
    constexpr Scope s = (S == Scope::Default) ? Scope::Device : S;
    if constexpr (O == Order::SeqCst) {
        if constexpr (s == Scope::Workgroup) asm volatile("fence.sc.cta;" ::: "memory");
        else if constexpr (s == Scope::Device) asm volatile("fence.sc.gpu;" ::: "memory");
        else asm volatile("fence.sc.sys;" ::: "memory");
    } else {
        if constexpr (s == Scope::Workgroup) asm volatile("fence.acq_rel.cta;" ::: "memory");
        else if constexpr (s == Scope::Device) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        else asm volatile("fence.acq_rel.sys;" ::: "memory");
    }
}

namespace detail {

// Validation rules of @access (src/macros.jl:217-233).
template <Scope S, Order O, bool IsLoad>
struct AccessCheck {
    static_assert(O != Order::AcqRel && O != Order::SeqCst,
                  "AcqRel and SeqCst are not valid orderings for loads and stores; use fence() instead.");
    static_assert(!(S != Scope::Default && (O == Order::Weak || O == Order::Volatile)),
                  "Weak and Volatile operations are scope-less: do not give a scope.");
    static_assert(!IsLoad || O != Order::Release, "Release is a store ordering.");
    static_assert(IsLoad || O != Order::Acquire, "Acquire is a load ordering.");
    static constexpr Order order = (O == Order::Default) ? (IsLoad ? Order::Acquire : Order::Release) : O;
    static constexpr Scope scope = (S == Scope::Default) ? Scope::Device : S;
};

// One PTX load/store per (ordering, scope, type).  The 8/16-bit types travel in 32-bit
// registers exactly as the reference's "r" constraints do (ext/CUDA/scopes_ordering.jl:68-86).
#define KI_LD_CASE(TY, PTXT, CONS, REGT)                                                              \
    template <Order O, Scope S>                                                                       \
    __device__ __forceinline__ TY ld_impl(const TY* p, TY*) {                                         \
        REGT r;                                                                                       \
        if constexpr (O == Order::Weak)                                                               \
            asm volatile("ld.weak.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory");      \
        else if constexpr (O == Order::Volatile)                                                      \
            asm volatile("ld.volatile.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory");  \
        else if constexpr (O == Order::Relaxed && S == Scope::Workgroup)                              \
            asm volatile("ld.relaxed.cta.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory"); \
        else if constexpr (O == Order::Relaxed && S == Scope::Device)                                 \
            asm volatile("ld.relaxed.gpu.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory"); \
        else if constexpr (O == Order::Relaxed)                                                       \
            asm volatile("ld.relaxed.sys.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory"); \
        else if constexpr (S == Scope::Workgroup)                                                     \
            asm volatile("ld.acquire.cta.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory"); \
        else if constexpr (S == Scope::Device)                                                        \
            asm volatile("ld.acquire.gpu.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory"); \
        else                                                                                          \
            asm volatile("ld.acquire.sys.global." PTXT " %0, [%1];" : "=" CONS(r) : "l"(p) : "memory"); \
        return (TY)r;                                                                                 \
    }                                                                                                 \
    template <Order O, Scope S>                                                                       \
    __device__ __forceinline__ void st_impl(TY* p, TY v) {                                            \
        REGT r = (REGT)v;                                                                             \
        if constexpr (O == Order::Weak)                                                               \
            asm volatile("st.weak.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");           \
        else if constexpr (O == Order::Volatile)                                                      \
            asm volatile("st.volatile.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");       \
        else if constexpr (O == Order::Relaxed && S == Scope::Workgroup)                              \
            asm volatile("st.relaxed.cta.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");    \
        else if constexpr (O == Order::Relaxed && S == Scope::Device)                                 \
            asm volatile("st.relaxed.gpu.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");    \
        else if constexpr (O == Order::Relaxed)                                                       \
            asm volatile("st.relaxed.sys.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");    \
        else if constexpr (S == Scope::Workgroup)                                                     \
            asm volatile("st.release.cta.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");    \
        else if constexpr (S == Scope::Device)                                                        \
            asm volatile("st.release.gpu.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");    \
        else                                                                                          \
            asm volatile("st.release.sys.global." PTXT " [%0], %1;" ::"l"(p), CONS(r) : "memory");    \
    }

#define KI_R(x) "r"(x)
#define KI_L(x) "l"(x)
#define KI_F(x) "f"(x)
#define KI_D(x) "d"(x)
KI_LD_CASE(int8_t, "s8", KI_R, int32_t)
KI_LD_CASE(uint8_t, "u8", KI_R, uint32_t)
KI_LD_CASE(int16_t, "s16", KI_R, int32_t)
KI_LD_CASE(uint16_t, "u16", KI_R, uint32_t)
KI_LD_CASE(int32_t, "s32", KI_R, int32_t)
KI_LD_CASE(uint32_t, "u32", KI_R, uint32_t)
KI_LD_CASE(float, "f32", KI_F, float)
KI_LD_CASE(int64_t, "s64", KI_L, int64_t)
KI_LD_CASE(uint64_t, "u64", KI_L, uint64_t)
KI_LD_CASE(double, "f64", KI_D, double)
#undef KI_LD_CASE

}  // namespace detail

// @access load: default ordering Acquire, default scope Device (src/macros.jl:235-246,268-275).
template <Order O = Order::Default, Scope S = Scope::Default, class T>
__device__ __forceinline__ T load(const T* p) {
    using C = detail::AccessCheck<S, O, true>;
    return detail::ld_impl<C::order, C::scope>(p, (T*)nullptr);
}

// @access store: default ordering Release, default scope Device (src/macros.jl:259-266).
template <Order O = Order::Default, Scope S = Scope::Default, class T>
__device__ __forceinline__ void store(T* p, T v) {
    using C = detail::AccessCheck<S, O, false>;
    detail::st_impl<C::order, C::scope>(p, v);
}

// ---------------------------------------------------------------------------------------------
// Lane / warp size (ext/KernelIntrinsicsCUDAExt.jl:13-19)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ int warpsize() { return kWarpSize; }
// 1-based lane index, like @laneid.
__device__ __forceinline__ int laneid() {
    unsigned l;
    asm("mov.u32 %0, %%laneid;" : "=r"(l));
    return (int)l + 1;
}
__device__ __forceinline__ unsigned lane0() {
    unsigned l;
    asm("mov.u32 %0, %%laneid;" : "=r"(l));
    return l;
}

// ---------------------------------------------------------------------------------------------
// @shfl on any trivially copyable type (src/warp.jl:114-158)
//
// The reference decomposes a value recursively into 32-bit words (8/16-bit types widened,
// 64/128-bit split hi/lo, structs field-wise, tuples element-wise) and shuffles each word.
// Here the value's bytes are viewed as ceil(sizeof(T)/4) 32-bit words and each is shuffled;
// for every field of every value this moves the same bits.
// Idx takes a 0-based source lane at this level; the 1-based host mirror subtracts one.
// ---------------------------------------------------------------------------------------------
enum class Dir { Up, Down, Xor, Idx };

template <Dir D>
__device__ __forceinline__ uint32_t shfl_word(uint32_t w, int src, unsigned mask) {
    if constexpr (D == Dir::Up) return __shfl_up_sync(mask, w, src, kWarpSize);
    else if constexpr (D == Dir::Down) return __shfl_down_sync(mask, w, src, kWarpSize);
    else if constexpr (D == Dir::Xor) return __shfl_xor_sync(mask, w, src, kWarpSize);
    else return __shfl_sync(mask, w, src, kWarpSize);
}

template <Dir D, class T>
__device__ __forceinline__ T shfl(T v, int src, unsigned mask = 0xffffffffu) {
    static_assert(std::is_trivially_copyable<T>::value, "shfl needs a trivially copyable type");
    constexpr int NW = (int)((sizeof(T) + 3) / 4);
    uint32_t w[NW];
    w[NW - 1] = 0;
    memcpy(w, &v, sizeof(T));
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = shfl_word<D>(w[i], src, mask);
    T r;
    memcpy(&r, w, sizeof(T));
    return r;
}

// ---------------------------------------------------------------------------------------------
// @warpreduce: inclusive scan with Up shuffles, offsets 1,2,..,16; the 1-based lane combines
// only when lane > offset (src/warp.jl:226-237).  op(shuffled, val) order is kept.
// ---------------------------------------------------------------------------------------------
template <class T, class Op>
__device__ __forceinline__ T warpreduce(T v, Op op, unsigned mask = 0xffffffffu) {
    const int lane = laneid();
#pragma unroll
    for (int offset = 1; offset < kWarpSize; offset <<= 1) {
        T s = shfl<Dir::Up>(v, offset, mask);
        if (lane > offset) v = op(s, v);
    }
    return v;
}

// @warpfold as written in the reference: Down shuffles; lane 1 holds the total, other lanes
// hold partial folds (src/warp.jl:273-282).
template <class T, class Op>
__device__ __forceinline__ T warpfold_down(T v, Op op) {
#pragma unroll
    for (int offset = 1; offset < kWarpSize; offset <<= 1) {
        T s = shfl<Dir::Down>(v, offset);
        v = op(s, v);
    }
    return v;
}

// Butterfly fold with xor shuffles: every lane holds the total.
template <class T, class Op>
__device__ __forceinline__ T warpfold(T v, Op op) {
#pragma unroll
    for (int offset = kWarpSize / 2; offset >= 1; offset >>= 1) {
        T s = shfl<Dir::Xor>(v, offset);
        v = op(s, v);
    }
    return v;
}

// ---------------------------------------------------------------------------------------------
// @vote (ext/CUDA/shuffle_vote.jl:23-34): vote.sync on CUDA; Ballot is a UInt32 mask,
// bit i (0-based) set when lane i's predicate holds.
// ---------------------------------------------------------------------------------------------
enum class Mode { All, AnyLane, Uni, Ballot };

__device__ __forceinline__ bool vote_all(bool p, unsigned mask = 0xffffffffu) { return __all_sync(mask, p); }
__device__ __forceinline__ bool vote_any(bool p, unsigned mask = 0xffffffffu) { return __any_sync(mask, p); }
__device__ __forceinline__ bool vote_uni(bool p, unsigned mask = 0xffffffffu) { return __uni_sync(mask, p); }
__device__ __forceinline__ uint32_t ballot(bool p, unsigned mask = 0xffffffffu) { return __ballot_sync(mask, p); }

// ---------------------------------------------------------------------------------------------
// Common binary operators
// ---------------------------------------------------------------------------------------------
struct Add {
    template <class T> __device__ __forceinline__ T operator()(T a, T b) const { return a + b; }
};
struct Max {
    template <class T> __device__ __forceinline__ T operator()(T a, T b) const { return a > b ? a : b; }
};
struct Min {
    template <class T> __device__ __forceinline__ T operator()(T a, T b) const { return a < b ? a : b; }
};
struct BitOr {
    template <class T> __device__ __forceinline__ T operator()(T a, T b) const { return a | b; }
};
struct BitAnd {
    template <class T> __device__ __forceinline__ T operator()(T a, T b) const { return a & b; }
};
struct BitXor {
    template <class T> __device__ __forceinline__ T operator()(T a, T b) const { return a ^ b; }
};

// Wrapping 64-bit add (Base.cumsum on Int64 wraps; signed overflow is UB in C++).
__device__ __forceinline__ int64_t wrap_add(int64_t a, int64_t b) {
    return (int64_t)((uint64_t)a + (uint64_t)b);
}
__device__ __forceinline__ int64_t wrap_sub(int64_t a, int64_t b) {
    return (int64_t)((uint64_t)a - (uint64_t)b);
}
struct WrapAdd {
    __device__ __forceinline__ int64_t operator()(int64_t a, int64_t b) const { return wrap_add(a, b); }
};

// ---------------------------------------------------------------------------------------------
// generate_partN as a compile-time table (src/vectorization.jl:306-338): for alignment residue
// r, the pieces (each a power of two, at most N/2 when misaligned, each naturally aligned).
// ---------------------------------------------------------------------------------------------
template <int N>
struct PartN {
    static_assert(N > 0 && (N & (N - 1)) == 0, "N must be a positive power of 2");
    int count[N];
    int piece[N][2 * 16 + 2];
    constexpr PartN() : count(), piece() {
        for (int r = 0; r < N; ++r) {
            if (r == 0) {
                count[0] = 1;
                piece[0][0] = N;
                continue;
            }
            int c = 0, remaining = N, pos = r;
            while (remaining > 0) {
                int max_load = N / 2;
                while (max_load > 0) {
                    if (pos % max_load == 0 && max_load <= remaining) break;
                    max_load /= 2;
                }
                if (max_load == 0) max_load = 1;
                piece[r][c++] = max_load;
                remaining -= max_load;
                pos = (pos + max_load) % N;
            }
            count[r] = c;
        }
    }
};

namespace detail {
// Naturally aligned load/store of B bytes (B a power of two); above 16 bytes, 16-byte pieces.
template <int B>
__device__ __forceinline__ void ld_aligned(const void* src, void* dst) {
    if constexpr (B == 1) *(uint8_t*)dst = *(const uint8_t*)src;
    else if constexpr (B == 2) *(uint16_t*)dst = *(const uint16_t*)src;
    else if constexpr (B == 4) *(uint32_t*)dst = *(const uint32_t*)src;
    else if constexpr (B == 8) *(uint2*)dst = *(const uint2*)src;
    else if constexpr (B == 16) *(uint4*)dst = *(const uint4*)src;
    else {
#pragma unroll
        for (int i = 0; i < B / 16; ++i) ((uint4*)dst)[i] = ((const uint4*)src)[i];
    }
}
template <int B>
__device__ __forceinline__ void st_aligned(void* dst, const void* src) {
    if constexpr (B == 1) *(uint8_t*)dst = *(const uint8_t*)src;
    else if constexpr (B == 2) *(uint16_t*)dst = *(const uint16_t*)src;
    else if constexpr (B == 4) *(uint32_t*)dst = *(const uint32_t*)src;
    else if constexpr (B == 8) *(uint2*)dst = *(const uint2*)src;
    else if constexpr (B == 16) *(uint4*)dst = *(const uint4*)src;
    else {
#pragma unroll
        for (int i = 0; i < B / 16; ++i) ((uint4*)dst)[i] = ((const uint4*)src)[i];
    }
}
template <class T, int N, int R, int P>
__device__ __forceinline__ void vload_piece(const T* a, T* out, int off) {
    constexpr PartN<N> tab{};
    if constexpr (P < tab.count[R]) {
        constexpr int len = tab.piece[R][P];
        ld_aligned<len * (int)sizeof(T)>(a + off, out + off);
        vload_piece<T, N, R, P + 1>(a, out, off + len);
    }
}
template <class T, int N, int R, int P>
__device__ __forceinline__ void vstore_piece(T* a, const T* in, int off) {
    constexpr PartN<N> tab{};
    if constexpr (P < tab.count[R]) {
        constexpr int len = tab.piece[R][P];
        st_aligned<len * (int)sizeof(T)>(a + off, in + off);
        vstore_piece<T, N, R, P + 1>(a, in, off + len);
    }
}
template <class T, int N, int R>
__device__ __forceinline__ void vload_dispatch(const T* a, T* out, int mod) {
    if constexpr (R < N) {
        if (mod == R) vload_piece<T, N, R, 0>(a, out, 0);
        else vload_dispatch<T, N, R + 1>(a, out, mod);
    }
}
template <class T, int N, int R>
__device__ __forceinline__ void vstore_dispatch(T* a, const T* in, int mod) {
    if constexpr (R < N) {
        if (mod == R) vstore_piece<T, N, R, 0>(a, in, 0);
        else vstore_dispatch<T, N, R + 1>(a, in, mod);
    }
}
}  // namespace detail

// vload_multi: N elements starting at element a[i] (i 0-based here), split into the naturally
// aligned pieces of generate_partN(N)[mod], mod = (ptr/sizeof(T) + i) % N
// (src/vectorization.jl:374-379).  Reads never leave [i, i+N).
template <class T, int N>
__device__ __forceinline__ void vload_multi(const T* a, int64_t i, T (&out)[N]) {
    static_assert((sizeof(T) & (sizeof(T) - 1)) == 0, "vload_multi needs a power-of-two element size");
    const int mod = (int)((((uintptr_t)a) / sizeof(T) + (uint64_t)i) % N);
    detail::vload_dispatch<T, N, 0>(a + i, out, mod);
}

// vstore_multi!: the store counterpart (src/vectorization.jl:407-420).
template <class T, int N>
__device__ __forceinline__ void vstore_multi(T* a, int64_t i, const T (&in)[N]) {
    static_assert((sizeof(T) & (sizeof(T) - 1)) == 0, "vstore_multi needs a power-of-two element size");
    const int mod = (int)((((uintptr_t)a) / sizeof(T) + (uint64_t)i) % N);
    detail::vstore_dispatch<T, N, 0>(a + i, in, mod);
}

// ---------------------------------------------------------------------------------------------
// Bounded waits.  Every spin in this library reads %globaltimer and gives up after a limit, so
// a wait on a flag that is never set ends with an error status instead of a hung GPU.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

}  // namespace ki
