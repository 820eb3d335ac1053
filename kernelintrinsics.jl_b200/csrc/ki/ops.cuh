// ki/ops.cuh -- the binary operators of the device-wide reduce and scan, with Julia Base semantics.
//
//   Add  sum / cumsum: integers wrap (two's complement); small integers widen as Base.add_sum
//        does (Int32 -> Int64, UInt32 -> UInt64); Float32 accumulates in Float64 and is rounded
//        back to Float32 once at the end (Base keeps Float32, within the documented tolerance).
//   Max  maximum / accumulate(max): a NaN operand wins, +0.0 is larger than -0.0 (Base.max).
//   Min  minimum / accumulate(min): a NaN operand wins, -0.0 is smaller than +0.0 (Base.min).
//   Mul  prod / cumprod: integers wrap; small integers widen as Base.mul_prod does (Int8/Int16/
//        Int32 -> Int64, UInt8/UInt16/UInt32 -> UInt64); Float32 multiplies in Float64 and is
//        rounded back to Float32 at the output.
//   Or, And, Xor  reduce(|, x) / accumulate(&, x) / xor over integers, in the input type.
// Sums widen Int8/Int16 and UInt8/UInt16 as Int32/UInt32 do (Base.add_sum).
//
// Traits<T, Op> gives the accumulation type A, the result type R, lift (T -> A), lower (A -> R),
// the identity of A and the operator on A.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <type_traits>

#include "../../../include/ki_b200.h"

namespace ki {

struct JAdd {};
struct JMax {};
struct JMin {};
struct JMul {};
struct JOr {};
struct JAnd {};
struct JXor {};

template <class Op>
struct IsBitwise : std::false_type {};
template <> struct IsBitwise<JOr> : std::true_type {};
template <> struct IsBitwise<JAnd> : std::true_type {};
template <> struct IsBitwise<JXor> : std::true_type {};

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
__device__ __forceinline__ T jmul(T a, T b) {
    if constexpr (std::is_integral<T>::value && sizeof(T) < 4) {  // no promotion to a signed int
        using U = typename std::make_unsigned<T>::type;
        return (T)(U)((uint32_t)(U)a * (uint32_t)(U)b);
    } else if constexpr (std::is_integral<T>::value) {
        using U = typename std::make_unsigned<T>::type;
        return (T)((U)a * (U)b);
    } else {
        return a * b;
    }
}

// Mul: the accumulation and result types of Add
template <class T>
struct Traits<T, JMul> {
    using A = typename Traits<T, JAdd>::A;
    using R = typename Traits<T, JAdd>::R;
    __host__ __device__ static __forceinline__ A lift(T x) { return (A)x; }
    __host__ __device__ static __forceinline__ R lower(A a) { return (R)a; }
    __device__ static __forceinline__ A identity() { return A(1); }
    __device__ static __forceinline__ A op(A a, A b) { return jmul(a, b); }
};

// Or / And / Xor: integers only, in the input type
template <class T, class Op>
struct BitTraits {
    static_assert(std::is_integral<T>::value, "bitwise operators take integers");
    using A = T;
    using R = T;
    __host__ __device__ static __forceinline__ A lift(T x) { return x; }
    __host__ __device__ static __forceinline__ R lower(A a) { return a; }
    __host__ __device__ static __forceinline__ A identity() { return std::is_same<Op, JAnd>::value ? (A)~A(0) : A(0); }
    __device__ static __forceinline__ A op(A a, A b) {
        if constexpr (std::is_same<Op, JOr>::value) return a | b;
        else if constexpr (std::is_same<Op, JAnd>::value) return a & b;
        else return a ^ b;
    }
};
template <class T>
struct Traits<T, JOr> : BitTraits<T, JOr> {};
template <class T>
struct Traits<T, JAnd> : BitTraits<T, JAnd> {};
template <class T>
struct Traits<T, JXor> : BitTraits<T, JXor> {};

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
// Compares and selects on the values themselves (NaN checks, then the signed-zero tie) were
// slower: Float32 accumulate(max) 0.62 -> 0.36 of the copy peak, Float64 0.52 -> 0.37, the
// Float32 / Float64 maximum reduce 1.01 -> 0.97.
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

// Element maps applied before a fold or a predicate (mapreduce(f, op, x), filter(v -> f(v) > t, x)),
// in the element type as Base computes them: abs wraps at the lowest signed value
// (abs(typemin(Int8)) == typemin(Int8)) and is the identity on unsigned types; abs2 is x*x with
// integer wrap-around; float abs clears the sign bit.
struct MapId {
    template <class T>
    __device__ static __forceinline__ T apply(T x) { return x; }
};
struct MapAbs {
    template <class T>
    __device__ static __forceinline__ T apply(T x) {
        if constexpr (std::is_floating_point<T>::value) return fabs(x);
        else if constexpr (std::is_unsigned<T>::value) return x;
        else if constexpr (sizeof(T) < 4) {
            // |x| in 32 bits, then truncated to T (which wraps typemin back to itself, as Base's abs
            // does).  Written as a 16-bit abs, the compiler returned +32768 for Int16 -32768 once the
            // value was widened for the sum; the 32-bit abs goes through inline PTX so that the
            // truncation is kept.
            int32_t a;
            asm("abs.s32 %0, %1;" : "=r"(a) : "r"((int32_t)x));
            return (T)a;
        } else {
            using U = typename std::make_unsigned<T>::type;
            return x < 0 ? (T)(U)(U(0) - (U)x) : x;
        }
    }
};
struct MapAbs2 {
    template <class T>
    __device__ static __forceinline__ T apply(T x) { return jmul(x, x); }
};

// The identity of Op as an element of T (what pads a partial tile).
template <class T, class Op>
__device__ __forceinline__ T pad_value() {
    if constexpr (std::is_same<Op, JAdd>::value || std::is_same<Op, JOr>::value || std::is_same<Op, JXor>::value)
        return T(0);
    else if constexpr (std::is_same<Op, JMul>::value) return T(1);
    else if constexpr (std::is_same<Op, JAnd>::value) return (T)~T(0);
    else if constexpr (std::is_same<Op, JMax>::value) return lowest_of<T>();
    else return highest_of<T>();
}

// Calls f(T{}) for the element type an ABI dtype code names (KI_I8 ... KI_F64); bad for another code.
template <class F>
inline int with_dtype(int dtype, int bad, F&& f) {
    switch (dtype) {
        case KI_I8: return f(int8_t{});
        case KI_U8: return f(uint8_t{});
        case KI_I16: return f(int16_t{});
        case KI_U16: return f(uint16_t{});
        case KI_I32: return f(int32_t{});
        case KI_U32: return f(uint32_t{});
        case KI_I64: return f(int64_t{});
        case KI_U64: return f(uint64_t{});
        case KI_F32: return f(float{});
        case KI_F64: return f(double{});
        default: return bad;
    }
}

// Whether Op is defined on T (the bitwise operators take integers only).
template <class T, class Op>
constexpr bool op_takes() {
    return std::is_integral<T>::value || !IsBitwise<Op>::value;
}

// 16-byte vector of T.
template <class T>
struct alignas(16) Vec16 {
    T v[16 / sizeof(T)];
};

// 16 bytes of T kept as four 32-bit words, elements taken out on use.  An array of sixteen 1-byte
// elements would occupy sixteen registers; this keeps four whatever the element size.
template <class T>
struct Packed16 {
    uint4 raw;
    static constexpr int kN = (int)(16 / sizeof(T));
    __device__ __forceinline__ uint32_t word(int k) const { return k == 0 ? raw.x : k == 1 ? raw.y : k == 2 ? raw.z : raw.w; }
    __device__ __forceinline__ void set_word(int k, uint32_t v) {
        if (k == 0) raw.x = v;
        else if (k == 1) raw.y = v;
        else if (k == 2) raw.z = v;
        else raw.w = v;
    }
    __device__ __forceinline__ T get(int e) const {
        T x;
        if constexpr (sizeof(T) == 8) {
            const uint64_t b = ((uint64_t)word(2 * e + 1) << 32) | word(2 * e);
            memcpy(&x, &b, 8);
        } else if constexpr (sizeof(T) == 4) {
            const uint32_t b = word(e);
            memcpy(&x, &b, 4);
        } else {
            using U = typename std::make_unsigned<T>::type;
            constexpr int kPerWord = (int)(4 / sizeof(T));
            x = (T)(U)(word(e / kPerWord) >> (8 * sizeof(T) * (e % kPerWord)));
        }
        return x;
    }
    __device__ __forceinline__ void set(int e, T x) {
        if constexpr (sizeof(T) == 8) {
            uint64_t b;
            memcpy(&b, &x, 8);
            set_word(2 * e, (uint32_t)b);
            set_word(2 * e + 1, (uint32_t)(b >> 32));
        } else if constexpr (sizeof(T) == 4) {
            uint32_t b;
            memcpy(&b, &x, 4);
            set_word(e, b);
        } else {
            using U = typename std::make_unsigned<T>::type;
            constexpr int kPerWord = (int)(4 / sizeof(T));
            const int sh = 8 * (int)sizeof(T) * (e % kPerWord);
            const uint32_t m = (uint32_t)(U)~U(0) << sh;
            set_word(e / kPerWord, (word(e / kPerWord) & ~m) | (((uint32_t)(U)x << sh) & m));
        }
    }
};

#ifndef KI_SWAR
#define KI_SWAR 1
#endif
#ifndef KI_SWAR16_MAXMIN
#define KI_SWAR16_MAXMIN 1
#endif
#ifndef KI_SWAR8_MAXMIN
#define KI_SWAR8_MAXMIN 1
#endif
#ifndef KI_SWAR8_SPLIT
#define KI_SWAR8_SPLIT 1
#endif
// 1- and 2-byte elements whose scan or reduce keeps the element type (|, & and xor; max and min where the
// byte or halfword SIMD form pays): four or two elements per 32-bit word at once (SWAR).  comb
// combines the element lanes of two words; kId is the operator's identity in every lane.  A word's
// inclusive prefix takes one shifted combine per doubling; a lane's four words are chained by
// broadcasting each word's last element.  With all 8 rows of a warp's span in flight (the generic
// path takes 2 at a time) this took UInt8 accumulate(|), (&), (xor) from 0.44-0.46 to 0.61 of the
// copy peak at 2^28.  Byte max / min: with __vmaxs4 / __vmins4, Int8 0.29 -> 0.34-0.35 (__vmaxu4 for
// UInt8 was slower than element by element, 0.38 -> 0.35); through the halfword instructions below
// (SwarBytePair) Int8 0.42, UInt8 0.46-0.47, and with the scan keeping the words split until the
// running prefix is in, Int8 0.465, UInt8 0.51-0.53, results identical.
// Halfwords (Int16 / UInt16, __vmaxs2 / __vmaxu2 / __vmins2 / __vminu2 for max / min): |, &, xor
// 0.66 -> 0.77-0.79, max / min 0.61-0.62 -> 0.75-0.77.
template <class T, class Op>
struct Swar {
    static constexpr bool kOn = false;
};
template <class T, class Op, uint32_t ID>
struct SwarBase {
    static_assert(sizeof(T) == 1 || sizeof(T) == 2, "byte or halfword lanes");
    static constexpr bool kOn = KI_SWAR != 0;
    static constexpr int kBits = 8 * (int)sizeof(T);                      // bits per element
    static constexpr uint32_t kRep = sizeof(T) == 1 ? 0x01010101u : 0x00010001u;
    static constexpr uint32_t kMask = sizeof(T) == 1 ? 0xFFu : 0xFFFFu;
    static constexpr uint32_t kId = ID * kRep;
    static constexpr bool kOwnPrefix = false;  // true where the operator has its own word prefix
    static constexpr bool kSplit = false;      // true where scans keep the words split (byte max / min)
    __device__ static __forceinline__ uint32_t bcast(uint32_t e) { return (e & kMask) * kRep; }
    // the word's last element in every lane (one byte permute)
    __device__ static __forceinline__ uint32_t top(uint32_t w) {
        return __byte_perm(w, 0u, sizeof(T) == 1 ? 0x3333u : 0x3232u);
    }
    // element lane r of w in every lane
    __device__ static __forceinline__ uint32_t spread(uint32_t w, int r) {
        return __byte_perm(w, 0u, sizeof(T) == 1 ? 0x1111u * (uint32_t)r : (r ? 0x3232u : 0x1010u));
    }
};
template <class T>
struct Swar<T, JOr> : SwarBase<T, JOr, 0x00u> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return a | b; }
};
template <class T>
struct Swar<T, JAnd> : SwarBase<T, JAnd, (sizeof(T) == 1 ? 0xFFu : 0xFFFFu)> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return a & b; }
};
template <class T>
struct Swar<T, JXor> : SwarBase<T, JXor, 0x00u> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return a ^ b; }
};
#if KI_SWAR8_MAXMIN
// Byte max / min through the halfword max / min instructions (max.s16x2 and the like, sm_90 and
// later): for two halfwords whose high bytes are elements x and y, the larger (smaller) halfword has
// the larger (smaller) of x and y as its high byte whatever the low bytes hold, since a low byte moves
// a halfword by less than one step of its high byte.  So the odd bytes of a word take one halfword
// instruction as they lie, the even bytes one after a shift by 8, and a byte permute puts the high
// bytes back in place.  A word's inclusive prefix p0..p3 of bytes b0..b3 is four halfword
// instructions: m = op(b0,b1) | op(b2,b3) (high bytes), s = m moved up a halfword over the identity,
// op(m, s) = p1 | p3 and op(b0 | b2, s) = p0 | p2.
template <class T, class Op, uint32_t ID>
struct SwarBytePair : SwarBase<T, Op, ID> {
    static constexpr bool kOwnPrefix = true;
    static constexpr bool kSplit = KI_SWAR8_SPLIT != 0;
    __device__ static __forceinline__ uint32_t h(uint32_t a, uint32_t b) {
        uint32_t d;
        if constexpr (std::is_same<Op, JMax>::value && std::is_signed<T>::value)
            asm("max.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        else if constexpr (std::is_same<Op, JMax>::value)
            asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        else if constexpr (std::is_signed<T>::value)
            asm("min.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        else
            asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) {
        return __byte_perm(h(a << 8, b << 8), h(a, b), 0x7351u);
    }
    // the prefix in split form: pe holds p0 | p2 and po p1 | p3 in the high bytes of its halfwords
    __device__ static __forceinline__ void prefix_split(uint32_t w, uint32_t& pe, uint32_t& po) {
        const uint32_t e = w << 8;                   // high bytes b0 | b2
        const uint32_t m = h(e, w);                  // high bytes op(b0,b1) | op(b2,b3)
        const uint32_t s = (m << 16) | (ID * 0x0101u);
        pe = h(e, s);
        po = h(m, s);
    }
    __device__ static __forceinline__ uint32_t join(uint32_t pe, uint32_t po) { return __byte_perm(pe, po, 0x7351u); }
    __device__ static __forceinline__ uint32_t prefix(uint32_t w) {
        uint32_t pe, po;
        prefix_split(w, pe, po);
        return join(pe, po);
    }
    // chains a split prefix onto the split prefix before it (whose last element is po_prev's top byte)
    __device__ static __forceinline__ void chain(uint32_t& pe, uint32_t& po, uint32_t po_prev) {
        const uint32_t c = __byte_perm(po_prev, 0u, 0x3333u);
        pe = h(pe, c);
        po = h(po, c);
    }
    // op over the 16 bytes of r into the split accumulators (order does not matter for max / min)
    __device__ static __forceinline__ void fold16(uint4 r, uint32_t& ae, uint32_t& ao) {
        ao = h(ao, h(h(r.x, r.y), h(r.z, r.w)));
        ae = h(ae, h(h(r.x << 8, r.y << 8), h(r.z << 8, r.w << 8)));
    }
    __device__ static __forceinline__ uint32_t fold_total(uint32_t ae, uint32_t ao) {
        const uint32_t t = h(ae, ao);  // high bytes: the totals of the two halves
        return h(t, t << 16) >> 24;
    }
};
template <>
struct Swar<int8_t, JMax> : SwarBytePair<int8_t, JMax, 0x80u> {};
template <>
struct Swar<int8_t, JMin> : SwarBytePair<int8_t, JMin, 0x7Fu> {};
template <>
struct Swar<uint8_t, JMax> : SwarBytePair<uint8_t, JMax, 0x00u> {};
template <>
struct Swar<uint8_t, JMin> : SwarBytePair<uint8_t, JMin, 0xFFu> {};
#else
template <>
struct Swar<int8_t, JMax> : SwarBase<int8_t, JMax, 0x80u> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return __vmaxs4(a, b); }
};
template <>
struct Swar<int8_t, JMin> : SwarBase<int8_t, JMin, 0x7Fu> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return __vmins4(a, b); }
};
#endif
#if KI_SWAR16_MAXMIN
template <>
struct Swar<int16_t, JMax> : SwarBase<int16_t, JMax, 0x8000u> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return __vmaxs2(a, b); }
};
template <>
struct Swar<int16_t, JMin> : SwarBase<int16_t, JMin, 0x7FFFu> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return __vmins2(a, b); }
};
template <>
struct Swar<uint16_t, JMax> : SwarBase<uint16_t, JMax, 0x0000u> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return __vmaxu2(a, b); }
};
template <>
struct Swar<uint16_t, JMin> : SwarBase<uint16_t, JMin, 0xFFFFu> {
    __device__ static __forceinline__ uint32_t comb(uint32_t a, uint32_t b) { return __vminu2(a, b); }
};
#endif
// only for 1- and 2-byte elements whose result keeps the type
template <class T, class Op>
constexpr bool swar_on() {
    if constexpr (sizeof(T) <= 2 && std::is_same<typename Traits<T, Op>::R, T>::value) return Swar<T, Op>::kOn;
    else return false;
}
// inclusive prefix of the element lanes of w (lowest lane first)
template <class SW>
__device__ __forceinline__ uint32_t swar_prefix(uint32_t w) {
    if constexpr (SW::kOwnPrefix) {
        return SW::prefix(w);
    } else {
#pragma unroll
        for (int s = SW::kBits; s < 32; s <<= 1) w = SW::comb(w, (w << s) | (SW::kId & ((1u << s) - 1u)));
        return w;
    }
}

}  // namespace ki
