// ki/ops.cuh -- the binary operators of the device-wide reduce and scan, with Julia Base semantics.
//
//   Add  sum / cumsum: integers wrap (two's complement); small integers widen as Base.add_sum
//        does (Int32 -> Int64, UInt32 -> UInt64); Float32 accumulates in Float64 and is rounded
//        back to Float32 once at the end (Base keeps Float32, within the documented tolerance).
//   Max  maximum / accumulate(max): a NaN operand wins, +0.0 is larger than -0.0 (Base.max).
//   Min  minimum / accumulate(min): a NaN operand wins, -0.0 is smaller than +0.0 (Base.min).
//
// Traits<T, Op> gives the accumulation type A, the result type R and the identity of A.
#pragma once

#include <cstdint>
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

template <class T>
__device__ __forceinline__ T jmax(T a, T b) {
    if constexpr (std::is_floating_point<T>::value) {
        if (a != a) return a;
        if (b != b) return b;
        if (a == b) return signbit(a) ? b : a;  // +0.0 over -0.0
    }
    return a > b ? a : b;
}

template <class T>
__device__ __forceinline__ T jmin(T a, T b) {
    if constexpr (std::is_floating_point<T>::value) {
        if (a != a) return a;
        if (b != b) return b;
        if (a == b) return signbit(a) ? a : b;  // -0.0 under +0.0
    }
    return a < b ? a : b;
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

template <class T>
struct Traits<T, JMax> {
    using A = T;
    using R = T;
    __device__ static __forceinline__ A identity() { return lowest_of<T>(); }
    __device__ static __forceinline__ A op(A a, A b) { return jmax(a, b); }
};

template <class T>
struct Traits<T, JMin> {
    using A = T;
    using R = T;
    __device__ static __forceinline__ A identity() { return highest_of<T>(); }
    __device__ static __forceinline__ A op(A a, A b) { return jmin(a, b); }
};

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
