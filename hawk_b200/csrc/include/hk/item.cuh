// hawk_b200 device library: small fixed-size vectors and matrices.
//
// The emitted body (the reference renderer's text, hawk/emit/render.py:140,
// spelled by the reference's writer, hawk/emit/writer_aether.py:1120-1180)
// names a rank-1 value ``Item<Real, N>`` and a rank-2 one ``Item<Real, R, C>``,
// builds them with brace lists, and combines them with infix operators and the
// methods ``dot``, ``norm``, ``sum``, ``transpose``, ``cwiseMul``, ``cross``
// and the free functions ``outer``, ``constant<extents<...>>``, ``select`` and
// the ``cwise*`` family.  Those names are the writer's, so they are kept; the
// types here are plain register-resident aggregates evaluated eagerly, one
// component at a time, which is the same arithmetic per component as a lazy
// expression would do.  Reductions run in ascending component order
// (``dot``: ((a0*b0 + a1*b1) + a2*b2) + ...), a division by a scalar is a
// multiplication by its reciprocal (the operation order the reference restates
// for the same library in hawk/embedded/writer.py:640-643), and a matrix
// product is a row-by-column ``dot``.
#pragma once
#include "base.cuh"
#include "math.cuh"

namespace hk {

template <class T, int... D> struct Item;

template <int... D> struct extents {};

// ---------------------------------------------------------------- rank 1
template <class T, int N>
struct Item<T, N> {
    T v[N];

    HK_FI T& operator[](int k) { return v[k]; }
    HK_FI const T& operator[](int k) const { return v[k]; }
    HK_FI T& operator()(int k) { return v[k]; }
    HK_FI const T& operator()(int k) const { return v[k]; }
    HK_FI T& at(int k) { return v[k]; }
    HK_FI const T& at(int k) const { return v[k]; }
    HK_FI T* data() { return v; }
    HK_FI const T* data() const { return v; }
    HK_FI const Item& get() const { return *this; }
    HK_FI const Item& eval() const { return *this; }
    HK_FI Item operator()() const { return *this; }      // a Mutable read's value: plane[i].get()()
    // component K of a Mutable read's value, as the body spells it: plane_i.eval<K>(i)
    template <int K, class I> HK_FI T eval(const I&) const { return v[K]; }
    static HK_HD constexpr int size() { return N; }

    HK_FI T dot(const Item& o) const {
        T s = v[0] * o.v[0];
#pragma unroll
        for (int k = 1; k < N; ++k) s = s + v[k] * o.v[k];
        return s;
    }
    HK_FI T squaredNorm() const { return dot(*this); }
    HK_FI T norm() const { return math::sqrt(dot(*this)); }
    HK_FI T sum() const {
        T s = v[0];
#pragma unroll
        for (int k = 1; k < N; ++k) s = s + v[k];
        return s;
    }
    HK_FI Item cwiseMul(const Item& o) const {
        Item r;
#pragma unroll
        for (int k = 0; k < N; ++k) r.v[k] = v[k] * o.v[k];
        return r;
    }
    HK_FI Item cross(const Item& o) const {
        static_assert(N == 3, "cross is defined for 3-vectors");
        return Item{{v[1] * o.v[2] - v[2] * o.v[1],
                     v[2] * o.v[0] - v[0] * o.v[2],
                     v[0] * o.v[1] - v[1] * o.v[0]}};
    }
};

// ---------------------------------------------------------------- rank 2
template <class T, int R, int C>
struct Item<T, R, C> {
    T m[R][C];

    HK_FI T& operator()(int r, int c) { return m[r][c]; }
    HK_FI const T& operator()(int r, int c) const { return m[r][c]; }
    HK_FI T& at(int r, int c) { return m[r][c]; }
    HK_FI const T& at(int r, int c) const { return m[r][c]; }
    HK_FI T* data() { return &m[0][0]; }
    HK_FI const T* data() const { return &m[0][0]; }
    HK_FI const Item& get() const { return *this; }
    HK_FI const Item& eval() const { return *this; }
    HK_FI Item operator()() const { return *this; }

    HK_FI Item<T, C, R> transpose() const {
        Item<T, C, R> t;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < C; ++c) t.m[c][r] = m[r][c];
        return t;
    }
    HK_FI T sum() const {
        T s = m[0][0];
#pragma unroll
        for (int k = 1; k < R * C; ++k) s = s + m[k / C][k % C];
        return s;
    }
    HK_FI Item cwiseMul(const Item& o) const {
        Item t;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < C; ++c) t.m[r][c] = m[r][c] * o.m[r][c];
        return t;
    }
};

// ---------------------------------------------------------------- elementwise helpers
namespace detail {
template <class T, int N, class F>
HK_FI Item<T, N> map1(const Item<T, N>& a, F f) {
    Item<T, N> r;
#pragma unroll
    for (int k = 0; k < N; ++k) r.v[k] = f(a.v[k]);
    return r;
}
template <class T, int R, int C, class F>
HK_FI Item<T, R, C> map1(const Item<T, R, C>& a, F f) {
    Item<T, R, C> t;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int c = 0; c < C; ++c) t.m[r][c] = f(a.m[r][c]);
    return t;
}
template <class T, int N, class F>
HK_FI Item<T, N> map2(const Item<T, N>& a, const Item<T, N>& b, F f) {
    Item<T, N> r;
#pragma unroll
    for (int k = 0; k < N; ++k) r.v[k] = f(a.v[k], b.v[k]);
    return r;
}
template <class T, int R, int C, class F>
HK_FI Item<T, R, C> map2(const Item<T, R, C>& a, const Item<T, R, C>& b, F f) {
    Item<T, R, C> t;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int c = 0; c < C; ++c) t.m[r][c] = f(a.m[r][c], b.m[r][c]);
    return t;
}
struct Add { template <class T> HK_FI T operator()(T a, T b) const { return a + b; } };
struct Sub { template <class T> HK_FI T operator()(T a, T b) const { return a - b; } };
struct Mul { template <class T> HK_FI T operator()(T a, T b) const { return a * b; } };
struct Div { template <class T> HK_FI T operator()(T a, T b) const { return a / b; } };
template <class T> struct MulBy { T s; HK_FI T operator()(T a) const { return a * s; } };
template <class T> struct ByMul { T s; HK_FI T operator()(T a) const { return s * a; } };
}  // namespace detail

// Item +/- Item, Item * scalar, scalar * Item, Item / scalar.
template <class T, int... D>
HK_FI Item<T, D...> operator+(const Item<T, D...>& a, const Item<T, D...>& b) { return detail::map2(a, b, detail::Add{}); }
template <class T, int... D>
HK_FI Item<T, D...> operator-(const Item<T, D...>& a, const Item<T, D...>& b) { return detail::map2(a, b, detail::Sub{}); }
template <class T, int... D>
HK_FI Item<T, D...> operator*(const Item<T, D...>& a, T s) { return detail::map1(a, detail::MulBy<T>{s}); }
template <class T, int... D>
HK_FI Item<T, D...> operator*(T s, const Item<T, D...>& a) { return detail::map1(a, detail::ByMul<T>{s}); }
template <class T, int... D>
HK_FI Item<T, D...> operator/(const Item<T, D...>& a, T s) {
    const T inv = T(1) / s;
    return detail::map1(a, detail::MulBy<T>{inv});
}
template <class T, int... D>
HK_FI Item<T, D...> operator-(const Item<T, D...>& a) { return a * T(-1); }

// Matrix-vector and matrix-matrix products.
template <class T, int R, int C>
HK_FI Item<T, R> operator*(const Item<T, R, C>& a, const Item<T, C>& x) {
    Item<T, R> y;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        T s = a.m[r][0] * x.v[0];
#pragma unroll
        for (int c = 1; c < C; ++c) s = s + a.m[r][c] * x.v[c];
        y.v[r] = s;
    }
    return y;
}
template <class T, int R, int K, int C>
HK_FI Item<T, R, C> operator*(const Item<T, R, K>& a, const Item<T, K, C>& b) {
    Item<T, R, C> y;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int c = 0; c < C; ++c) {
            T s = a.m[r][0] * b.m[0][c];
#pragma unroll
            for (int k = 1; k < K; ++k) s = s + a.m[r][k] * b.m[k][c];
            y.m[r][c] = s;
        }
    return y;
}

template <class T, int R, int C>
HK_FI Item<T, R, C> outer(const Item<T, R>& a, const Item<T, C>& b) {
    Item<T, R, C> y;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int c = 0; c < C; ++c) y.m[r][c] = a.v[r] * b.v[c];
    return y;
}

// constant<extents<D...>>(x): every component x (a broadcast scalar).
template <class E, class T> struct Constant;
template <int... D, class T> struct Constant<extents<D...>, T> {
    static HK_FI Item<T, D...> make(T x) {
        Item<T, D...> y;
        T* p = y.data();
#pragma unroll
        for (int k = 0; k < (D * ...); ++k) p[k] = x;
        return y;
    }
};
template <class T> struct Constant<extents<>, T> {     // rank 0: the scalar itself
    static HK_FI T make(T x) { return x; }
};
template <class E, class T>
HK_FI auto constant(T x) -> decltype(Constant<E, T>::make(x)) { return Constant<E, T>::make(x); }

// select(c, a, b): a where c, else b; scalar or componentwise condition.
template <class T>
HK_FI T select(bool c, T a, T b) { return c ? a : b; }
template <class T, int... D>
HK_FI Item<T, D...> select(bool c, const Item<T, D...>& a, const Item<T, D...>& b) { return c ? a : b; }

// The componentwise math family.
#define HK_CWISE1(NAME, FN)                                                        \
    template <class T, int... D>                                                   \
    HK_FI Item<T, D...> NAME(const Item<T, D...>& a) {                             \
        return detail::map1(a, [](T x) { return math::FN(x); });                   \
    }
HK_CWISE1(cwiseAbs, abs)
HK_CWISE1(cwiseSqrt, sqrt)
HK_CWISE1(cwiseRsqrt, rsqrt)
HK_CWISE1(cwiseExp, exp)
HK_CWISE1(cwiseLog, log)
HK_CWISE1(cwiseSin, sin)
HK_CWISE1(cwiseCos, cos)
HK_CWISE1(cwiseAsin, asin)
HK_CWISE1(cwiseAcos, acos)
HK_CWISE1(cwiseAtan, atan)
HK_CWISE1(cwiseTan, tan)
HK_CWISE1(cwiseTanh, tanh)
#undef HK_CWISE1

#define HK_CWISE2(NAME, EXPR)                                                          \
    template <class T, int... D>                                                       \
    HK_FI Item<T, D...> NAME(const Item<T, D...>& a, const Item<T, D...>& b) {         \
        return detail::map2(a, b, [](T x, T y) { return EXPR; });                      \
    }                                                                                  \
    template <class T, int... D>                                                       \
    HK_FI Item<T, D...> NAME(const Item<T, D...>& a, T y) {                            \
        return detail::map1(a, [y](T x) { return EXPR; });                             \
    }
HK_CWISE2(cwiseMin, math::fmin(x, y))
HK_CWISE2(cwiseMax, math::fmax(x, y))
HK_CWISE2(cwiseDiv, x / y)
HK_CWISE2(cwisePow, math::pow(x, y))
#undef HK_CWISE2

}  // namespace hk
