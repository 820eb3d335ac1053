// ki/ops.cuh -- the binary operators of the device-wide reduce and scan, with Julia Base semantics.
//
//   Add  sum / cumsum: integers wrap (two's complement); small integers widen as Base.add_sum
//        does (Int32 -> Int64, UInt32 -> UInt64); Float32 accumulates in Float64 and is rounded
//        back to Float32 once at the end (Base keeps Float32, within the documented tolerance).
//   Max  maximum / accumulate(max): a NaN operand wins, +0.0 is larger than -0.0 (Base.max).
//   Min  minimum / accumulate(min): a NaN operand wins, -0.0 is smaller than +0.0 (Base.min).
//
// Traits<T, Op> gives the accumulation type A, the result type R, lift (T -> A), lower (A -> R),
// the identity of A and the operator on A.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <type_traits>

namespace ki {

struct JAdd {};
struct JMax {};
struct JMin {};

template <class T>
__device__ __forceinline__ T jadd(T a, T b) {
    if constexpr (std::is_integral<T>::value) {
        using U = typename std::make_unsigned<T>::type;
        return (T)((U)a + (U)b);
    } else {
        return a + b;
    }
}

// Base.max / Base.min for floats, as selects (no branches): a NaN operand wins and the sign bit
// orders equal zeros.
template <class T>
__device__ __forceinline__ T jmax(T x, T y) {
    if constexpr (std::is_floating_point<T>::value) {
        const bool take_y = (y > x) | (signbit(y) < signbit(x));
        const T yy = (x != x) ? x : y;
        const T xx = (y != y) ? y : x;
        return take_y ? yy : xx;
    } else {
        return x > y ? x : y;
    }
}

template <class T>
__device__ __forceinline__ T jmin(T x, T y) {
    if constexpr (std::is_floating_point<T>::value) {
        const bool take_y = (y < x) | (signbit(y) > signbit(x));
        const T yy = (x != x) ? x : y;
        const T xx = (y != y) ? y : x;
        return take_y ? yy : xx;
    } else {
        return x < y ? x : y;
    }
}

template <class T, class Op>
struct Traits;

// Add: widened or Float64 accumulation
template <class T>
struct Traits<T, JAdd> {
    using A = typename std::conditional<
        std::is_floating_point<T>::value, double,
        typename std::conditional<(sizeof(T) < 8),
                                  typename std::conditional<std::is_signed<T>::value, int64_t, uint64_t>::type,
                                  T>::type>::type;
    using R = typename std::conditional<std::is_same<T, float>::value, float, A>::type;
    __host__ __device__ static __forceinline__ A lift(T x) { return (A)x; }
    __host__ __device__ static __forceinline__ R lower(A a) { return (R)a; }
    __device__ static __forceinline__ A identity() { return A(0); }
    __device__ static __forceinline__ A op(A a, A b) { return jadd(a, b); }
};

template <class T>
__device__ __forceinline__ T lowest_of() {
    if constexpr (std::is_floating_point<T>::value) return -INFINITY;
    else if constexpr (std::is_signed<T>::value) return (T)((typename std::make_unsigned<T>::type)1 << (8 * sizeof(T) - 1));
    else return T(0);
}
template <class T>
__device__ __forceinline__ T highest_of() {
    if constexpr (std::is_floating_point<T>::value) return INFINITY;
    else if constexpr (std::is_signed<T>::value) return (T)(~((typename std::make_unsigned<T>::type)1 << (8 * sizeof(T) - 1)));
    else return (T)~T(0);
}

// Order-preserving unsigned keys of a float (Base.isless order with -0.0 < +0.0).  A NaN maps to
// the key that wins (all ones for max, zero for min), so max/min of floats run as integer
// max/min: one instruction per step instead of Base.max's select chain.  Keys are converted back
// once, at the output (a NaN result comes back as the canonical quiet NaN).
template <class F>
struct FloatKey {
    using K = typename std::conditional<sizeof(F) == 4, uint32_t, uint64_t>::type;
    static constexpr K kSign = (K)1 << (8 * sizeof(F) - 1);
    __host__ __device__ static __forceinline__ K key(F x, bool for_max) {
        K b;
        memcpy(&b, &x, sizeof(F));
        if (x != x) return for_max ? (K)~(K)0 : (K)0;
        return (b & kSign) ? (K)~b : (K)(b | kSign);
    }
    __host__ __device__ static __forceinline__ F value(K k, bool for_max) {
        if (k == (for_max ? (K)~(K)0 : (K)0)) return F(NAN);
        const K b = (k & kSign) ? (K)(k & ~kSign) : (K)~k;
        F x;
        memcpy(&x, &b, sizeof(F));
        return x;
    }
};

template <class T, bool MAX>
struct MaxMinTraits {
    static constexpr bool kFloat = std::is_floating_point<T>::value;
    using A = typename std::conditional<kFloat, typename FloatKey<typename std::conditional<kFloat, T, float>::type>::K,
                                        T>::type;
    using R = T;
    __host__ __device__ static __forceinline__ A lift(T x) {
        if constexpr (kFloat) return FloatKey<T>::key(x, MAX);
        else return x;
    }
    __host__ __device__ static __forceinline__ R lower(A a) {
        if constexpr (kFloat) return FloatKey<T>::value(a, MAX);
        else return a;
    }
    __device__ static __forceinline__ A identity() {  // key of -Inf / +Inf; lowest / highest integer
        if constexpr (kFloat) return lift(MAX ? (T)-INFINITY : (T)INFINITY);
        else return MAX ? lowest_of<T>() : highest_of<T>();
    }
    __device__ static __forceinline__ A op(A a, A b) { return MAX ? (a > b ? a : b) : (a < b ? a : b); }
};

template <class T>
struct Traits<T, JMax> : MaxMinTraits<T, true> {};

template <class T>
struct Traits<T, JMin> : MaxMinTraits<T, false> {};

// Functor form for the warp folds and scans of ki/intrinsics.cuh.
template <class T, class Op>
struct OpFn {
    using A = typename Traits<T, Op>::A;
    __device__ __forceinline__ A operator()(A a, A b) const { return Traits<T, Op>::op(a, b); }
};

// 16-byte vector of T.
template <class T>
struct alignas(16) Vec16 {
    T v[16 / sizeof(T)];
};

}  // namespace ki
