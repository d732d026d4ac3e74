// hawk_b200 device library: integer-plane arithmetic.
//
// The body calls these as ``hawk_abi::int_<op>`` (hawk/emit/writer_aether.py:1311-1318
// routes every integer-plane op that could overflow or promote through them).
// Semantics are the language's (stated at hawk/emit/wrapper.py:846-853 and
// pinned against NumPy by tests/test_int_planes.py): two's-complement wrapping
// add/sub/mul/neg/abs; floor division and divisor-signed modulo, a zero divisor
// giving 0; shifts by a count outside [0, bits) giving 0 (-1 for a negative
// value shifted right); float -> integer truncating toward zero, saturating at
// the type's range, NaN -> 0.  The name is the one the body text spells.
#pragma once
#include "base.cuh"

namespace hawk_abi {

template <class T> struct int_traits;
template <> struct int_traits<int> {
    typedef unsigned int U;
    static constexpr bool is_signed = true;
    static constexpr int lo = -2147483647 - 1;
    static constexpr int hi = 2147483647;
    static constexpr unsigned bits = 32u;
};
template <> struct int_traits<unsigned int> {
    typedef unsigned int U;
    static constexpr bool is_signed = false;
    static constexpr unsigned int lo = 0u;
    static constexpr unsigned int hi = 4294967295u;
    static constexpr unsigned bits = 32u;
};
template <> struct int_traits<long long> {
    typedef unsigned long long U;
    static constexpr bool is_signed = true;
    static constexpr long long lo = -9223372036854775807LL - 1;
    static constexpr long long hi = 9223372036854775807LL;
    static constexpr unsigned bits = 64u;
};

template <class T> HK_HD T int_add(T a, T b) {
    typedef typename int_traits<T>::U U;
    return static_cast<T>(static_cast<U>(a) + static_cast<U>(b));
}
template <class T> HK_HD T int_sub(T a, T b) {
    typedef typename int_traits<T>::U U;
    return static_cast<T>(static_cast<U>(a) - static_cast<U>(b));
}
template <class T> HK_HD T int_mul(T a, T b) {
    typedef typename int_traits<T>::U U;
    return static_cast<T>(static_cast<U>(a) * static_cast<U>(b));
}
template <class T> HK_HD T int_neg(T a) {
    typedef typename int_traits<T>::U U;
    return static_cast<T>(U(0) - static_cast<U>(a));
}
template <class T> HK_HD T int_abs(T a) {
    if constexpr (int_traits<T>::is_signed) return a < T(0) ? int_neg(a) : a;
    else return a;
}
template <class T> HK_HD T int_min(T a, T b) { return b < a ? b : a; }
template <class T> HK_HD T int_max(T a, T b) { return a < b ? b : a; }
template <class T> HK_HD T int_clamp_index(T i, T n) {
    typedef typename int_traits<T>::U U;
    if (static_cast<U>(i) < static_cast<U>(n)) return i;
    return i < T(0) ? T(0) : static_cast<T>(n - T(1));
}
template <class T> HK_HD T int_floordiv(T a, T b) {
    if (b == T(0)) return T(0);
    if constexpr (int_traits<T>::is_signed) {
        if (b == T(-1)) return int_neg(a);
        const T q = static_cast<T>(a / b);
        const bool inexact = static_cast<T>(a % b) != T(0);
        return (inexact && ((a < T(0)) != (b < T(0)))) ? static_cast<T>(q - T(1)) : q;
    } else {
        return static_cast<T>(a / b);
    }
}
template <class T> HK_HD T int_mod(T a, T b) {
    if (b == T(0)) return T(0);
    if constexpr (int_traits<T>::is_signed) {
        if (b == T(-1)) return T(0);
        const T r = static_cast<T>(a % b);
        return (r != T(0) && ((r < T(0)) != (b < T(0)))) ? static_cast<T>(r + b) : r;
    } else {
        return static_cast<T>(a % b);
    }
}
template <class T> HK_HD T int_and(T a, T b) { return static_cast<T>(a & b); }
template <class T> HK_HD T int_or(T a, T b) { return static_cast<T>(a | b); }
template <class T> HK_HD T int_xor(T a, T b) { return static_cast<T>(a ^ b); }
template <class T> HK_HD T int_invert(T a) { return static_cast<T>(~a); }
template <class T> HK_HD T int_shl(T a, T b) {
    typedef typename int_traits<T>::U U;
    if (static_cast<U>(b) < static_cast<U>(int_traits<T>::bits))
        return static_cast<T>(static_cast<U>(a) << static_cast<U>(b));
    return T(0);
}
template <class T> HK_HD T int_shr(T a, T b) {
    typedef typename int_traits<T>::U U;
    if (static_cast<U>(b) < static_cast<U>(int_traits<T>::bits)) return static_cast<T>(a >> b);
    if constexpr (int_traits<T>::is_signed) return a < T(0) ? T(-1) : T(0);
    else return T(0);
}
template <class T, class R> HK_HD T int_from_real(R x) {
    if (x != x) return T(0);
    if (x <= static_cast<R>(int_traits<T>::lo)) return int_traits<T>::lo;
    if (x >= static_cast<R>(int_traits<T>::hi)) return int_traits<T>::hi;
    return static_cast<T>(x);
}

}  // namespace hawk_abi
