// hawk_b200 device library: per-lane (register-resident) linear algebra.
//
// The body spells a factorisation as a struct local filled in place and a solve
// as a call that writes its last operand (hawk/emit/writer_aether.py:551-622):
//     linalg::Cholesky<Real, 6> f;  linalg::cholesky<6>(f, A);
//     linalg::choSolve<1>(f, b, out);
// A and b are the sample's values (register Items, or plane proxies), ``out`` an
// Item or an output-plane proxy.  One thread holds one matrix (n <= 32,
// hawk/ir/linalg.py:33-36), every loop is unrolled, and the factor lives in
// registers.  The floating-point operation order is the one the reference
// restates, operation for operation, in hawk/embedded/linalg.py:188-300
// (factorisations) and :443-520 (solves): column-by-column Cholesky on the
// symmetric part (0.5*a_ij + 0.5*a_ji) with forward-ordered dot products,
// Crout LU with a first-of-equals pivot search, forward-ordered triangular
// sweeps; a failed factor (info > 0) solves to zeros.
#pragma once
#include "item.cuh"

namespace hk {
namespace linalg {

template <class T, int N> struct Cholesky {
    Item<T, N, N> l;
    int info;
};

template <class T, int N> struct Lu {
    Item<T, N, N> a;
    int piv[N];
    int info;
};

namespace detail {
// Element access over an Item, a proxy of a plane or anything with operator().
template <class V> HK_FI auto el(const V& v, int i) -> decltype(v(i)) { return v(i); }
template <class V> HK_FI auto el(const V& v, int i, int c) -> decltype(v(i, c)) { return v(i, c); }

template <class T, int N, int K> struct Rhs { typedef Item<T, N, K> type; };
template <class T, int N> struct Rhs<T, N, 1> { typedef Item<T, N> type; };

template <class T, int N, int K, class B>
HK_FI typename Rhs<T, N, K>::type load_rhs(const B& b) {
    typename Rhs<T, N, K>::type x;
    if constexpr (K == 1) {
#pragma unroll
        for (int i = 0; i < N; ++i) x(i) = static_cast<T>(el(b, i));
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
            for (int c = 0; c < K; ++c) x(i, c) = static_cast<T>(el(b, i, c));
    }
    return x;
}

template <class T, int N, int K, class O>
HK_FI void store_rhs(const typename Rhs<T, N, K>::type& x, O&& out) {
    if constexpr (K == 1) {
#pragma unroll
        for (int i = 0; i < N; ++i) out(i) = x(i);
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
            for (int c = 0; c < K; ++c) out(i, c) = x(i, c);
    }
}

}  // namespace detail

// L L^T = sym(A); info = first failing column (1-based), 0 on success.
template <int N, class T, class A>
HK_FI void cholesky(Cholesky<T, N>& f, const A& a) {
    f.info = 0;
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
        for (int c = 0; c < N; ++c) f.l.m[i][c] = T(0);
#pragma unroll
    for (int j = 0; j < N; ++j) {
        if (f.info == 0) {
            T d = (T(0.5) * static_cast<T>(detail::el(a, j, j))) + (T(0.5) * static_cast<T>(detail::el(a, j, j)));
#pragma unroll
            for (int k = 0; k < j; ++k) d = d - (f.l.m[j][k] * f.l.m[j][k]);
            if (d > T(0)) {
                const T ljj = math::sqrt(d);
                f.l.m[j][j] = ljj;
#pragma unroll
                for (int i = j + 1; i < N; ++i) {
                    T acc = (T(0.5) * static_cast<T>(detail::el(a, i, j))) + (T(0.5) * static_cast<T>(detail::el(a, j, i)));
#pragma unroll
                    for (int k = 0; k < j; ++k) acc = acc - (f.l.m[i][k] * f.l.m[j][k]);
                    f.l.m[i][j] = acc / ljj;
                }
            } else {
                f.info = j + 1;
            }
        }
    }
}

// The lower triangle of ``a`` taken as the factor; info = first column whose
// diagonal entry is not positive and finite, and then the factor is zero.
template <int N, class T, class A>
HK_FI void choleskyFrom(Cholesky<T, N>& f, const A& a) {
    f.info = 0;
#pragma unroll
    for (int j = 0; j < N; ++j) {
        const T d = static_cast<T>(detail::el(a, j, j));
        if (f.info == 0 && ((d <= T(0)) || !math::isfinite(d))) f.info = j + 1;
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
        for (int c = 0; c < N; ++c)
            f.l.m[i][c] = (f.info == 0 && c <= i) ? static_cast<T>(detail::el(a, i, c)) : T(0);
}

// x = A^{-1} b from the factor: forward sweep on L, backward sweep on L^T.
template <int K, class T, int N, class B, class O>
HK_FI void choSolve(const Cholesky<T, N>& f, const B& b, O&& out) {
    typename detail::Rhs<T, N, K>::type x = detail::load_rhs<T, N, K>(b);
    if (f.info == 0) {
#pragma unroll
        for (int c = 0; c < K; ++c) {
#pragma unroll
            for (int i = 0; i < N; ++i) {
                T acc = (K == 1) ? x.data()[i] : x.data()[i * K + c];
#pragma unroll
                for (int j = 0; j < i; ++j) acc = acc - (f.l.m[i][j] * x.data()[j * K + c]);
                x.data()[i * K + c] = acc / f.l.m[i][i];
            }
#pragma unroll
            for (int r = 0; r < N; ++r) {
                const int i = N - 1 - r;
                T acc = x.data()[i * K + c];
#pragma unroll
                for (int j = i + 1; j < N; ++j) acc = acc - (f.l.m[j][i] * x.data()[j * K + c]);
                x.data()[i * K + c] = acc / f.l.m[i][i];
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < N * K; ++k) x.data()[k] = T(0);
    }
    detail::store_rhs<T, N, K>(x, static_cast<O&&>(out));
}

// L y = b (forward sweep) and L^T y = b (backward sweep) against a factor's L.
template <int N2, int K, class T, int N, class B, class O>
HK_FI void triLower(const Item<T, N, N>& l, const B& b, O&& out) {
    typename detail::Rhs<T, N, K>::type x = detail::load_rhs<T, N, K>(b);
#pragma unroll
    for (int c = 0; c < K; ++c)
#pragma unroll
        for (int i = 0; i < N; ++i) {
            T acc = x.data()[i * K + c];
#pragma unroll
            for (int j = 0; j < i; ++j) acc = acc - (l.m[i][j] * x.data()[j * K + c]);
            x.data()[i * K + c] = acc / l.m[i][i];
        }
    detail::store_rhs<T, N, K>(x, static_cast<O&&>(out));
}

template <int N2, int K, class T, int N, class B, class O>
HK_FI void triUpperT(const Item<T, N, N>& l, const B& b, O&& out) {
    typename detail::Rhs<T, N, K>::type x = detail::load_rhs<T, N, K>(b);
#pragma unroll
    for (int c = 0; c < K; ++c)
#pragma unroll
        for (int r = 0; r < N; ++r) {
            const int i = N - 1 - r;
            T acc = x.data()[i * K + c];
#pragma unroll
            for (int j = i + 1; j < N; ++j) acc = acc - (l.m[j][i] * x.data()[j * K + c]);
            x.data()[i * K + c] = acc / l.m[i][i];
        }
    detail::store_rhs<T, N, K>(x, static_cast<O&&>(out));
}

// The factor as a matrix (its L; zeros for a failed factor).
template <class T, int N, class O>
HK_FI void choleskyFactor(const Cholesky<T, N>& f, O&& out) {
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
        for (int c = 0; c < N; ++c) out(i, c) = (f.info == 0) ? f.l.m[i][c] : T(0);
}

// P A = L U, Crout, column by column, pivot = first of equal magnitudes.
template <int N, class T, class A>
HK_FI void lu(Lu<T, N>& f, const A& a) {
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
        for (int c = 0; c < N; ++c) f.a.m[i][c] = static_cast<T>(detail::el(a, i, c));
    f.info = 0;
    if (N == 1) {
        f.piv[0] = 0;
        f.info = (f.a.m[0][0] != T(0)) ? 0 : 1;
        return;
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int m = (i < j) ? i : j;
            T acc = T(0);
#pragma unroll
            for (int k = 0; k < m; ++k) acc = acc + (f.a.m[i][k] * f.a.m[k][j]);
            f.a.m[i][j] = f.a.m[i][j] - acc;
        }
        int p = j;
        T big = math::abs(f.a.m[j][j]);
#pragma unroll
        for (int i = j + 1; i < N; ++i) {
            const T mag = math::abs(f.a.m[i][j]);
            if (mag > big) {
                big = mag;
                p = i;
            }
        }
        f.piv[j] = p;
        // p is a runtime row index: read and swap through a unrolled select so
        // the matrix stays in registers.
        T pj = f.a.m[j][j];
#pragma unroll
        for (int i = j + 1; i < N; ++i) if (p == i) pj = f.a.m[i][j];
        if (pj != T(0)) {
            if (p != j) {
#pragma unroll
                for (int i = j + 1; i < N; ++i) {
                    if (p == i) {
#pragma unroll
                        for (int c = 0; c < N; ++c) {
                            const T tmp = f.a.m[j][c];
                            f.a.m[j][c] = f.a.m[i][c];
                            f.a.m[i][c] = tmp;
                        }
                    }
                }
            }
            const T rcp = T(1) / f.a.m[j][j];
#pragma unroll
            for (int i = j + 1; i < N; ++i) f.a.m[i][j] = f.a.m[i][j] * rcp;
        } else if (f.info == 0) {
            f.info = j + 1;
        }
    }
}

namespace detail {
template <class T, int N, int K>
HK_FI void swap_rows(typename Rhs<T, N, K>::type& x, int a, int p) {
    // rows a and p (p >= a) exchanged, p a runtime index
#pragma unroll
    for (int i = 0; i < N; ++i) {
        if (i > a && p == i) {
#pragma unroll
            for (int c = 0; c < K; ++c) {
                const T tmp = x.data()[a * K + c];
                x.data()[a * K + c] = x.data()[i * K + c];
                x.data()[i * K + c] = tmp;
            }
        }
    }
}
}  // namespace detail

template <int K, class T, int N, class B, class O>
HK_FI void luSolve(const Lu<T, N>& f, const B& b, O&& out) {
    typename detail::Rhs<T, N, K>::type x = detail::load_rhs<T, N, K>(b);
    if (f.info == 0) {
        if (N > 1) {
#pragma unroll
            for (int k = 0; k < N; ++k) detail::swap_rows<T, N, K>(x, k, f.piv[k]);
        }
#pragma unroll
        for (int c = 0; c < K; ++c) {
            if (N > 1) {
#pragma unroll
                for (int i = 0; i < N; ++i) {
                    T acc = x.data()[i * K + c];
#pragma unroll
                    for (int j = 0; j < i; ++j) acc = acc - (f.a.m[i][j] * x.data()[j * K + c]);
                    x.data()[i * K + c] = acc;
                }
            }
#pragma unroll
            for (int r = 0; r < N; ++r) {
                const int i = N - 1 - r;
                T acc = x.data()[i * K + c];
#pragma unroll
                for (int j = i + 1; j < N; ++j) acc = acc - (f.a.m[i][j] * x.data()[j * K + c]);
                x.data()[i * K + c] = acc / f.a.m[i][i];
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < N * K; ++k) x.data()[k] = T(0);
    }
    detail::store_rhs<T, N, K>(x, static_cast<O&&>(out));
}

// det(A) from the factor: the product of U's diagonal, negated per row exchange
// as it is met (hawk/embedded/linalg.py:402-418); 0 for a failed factor.
template <class T, int N>
HK_FI T luDet(const Lu<T, N>& f) {
    T d = T(0);
    if (f.info == 0) {
        d = T(1);
#pragma unroll
        for (int k = 0; k < N; ++k) {
            d = d * f.a.m[k][k];
            if (f.piv[k] != k) d = -d;
        }
    }
    return d;
}

// ---------------------------------------------------------------- eigh

// Jacobi sweeps for dimension n (the count hawk/ir/linalg.py:82-84 records).
HK_HD constexpr int eigh_sweeps(int n) { return n <= 2 ? 2 : n <= 4 ? 6 : n <= 8 ? 8 : n <= 16 ? 12 : 15; }

template <class T> struct EighEps;
template <> struct EighEps<double> { static HK_HD constexpr double value() { return 2.220446049250313e-16; } };
template <> struct EighEps<float> { static HK_HD constexpr float value() { return 1.1920928955078125e-07f; } };

// w, V, info of the symmetric part of A: eigenvalues ascending, eigenvectors
// the columns of V (row-major v[i * N + j]), each signed so its first largest
// component is positive; info bit 1: the off-diagonal mass did not fall below
// (n eps)^2 of the Frobenius norm, bit 2: two eigenvalues closer than
// n eps |A|_F.  Cyclic Jacobi, operation for operation the order
// hawk/embedded/linalg.py:302-399 restates; the loops stay rolled (the
// matrix lives in the thread's local memory).
template <class T, int N> struct Eigh {
    T w[N];
    T v[N * N];
    int info;
};
template <class T, int N> struct EighValues {
    T w[N];
    T v[N * N];
    int info;
};

namespace detail {
template <int N, class T, class F, class A> HK_FI void eigh_into(F& f, const A& a, bool vectors) {
    const T zero = T(0), one = T(1), half = T(0.5);
    f.info = 0;
    if (N == 1) {
        f.w[0] = static_cast<T>(el(a, 0, 0));
        f.v[0] = one;
        return;
    }
    const T eps = EighEps<T>::value();
    T s[N][N];
    T fro2 = zero;
#pragma unroll 1
    for (int i = 0; i < N; ++i)
#pragma unroll 1
        for (int c = 0; c < N; ++c) f.v[i * N + c] = zero;
#pragma unroll 1
    for (int i = 0; i < N; ++i) {
#pragma unroll 1
        for (int j = 0; j < N; ++j) {
            if (j >= i) s[i][j] = (half * static_cast<T>(el(a, i, j))) + (half * static_cast<T>(el(a, j, i)));
            else s[i][j] = s[j][i];
            fro2 = fro2 + (s[i][j] * s[i][j]);
        }
        f.v[i * N + i] = one;
    }
#pragma unroll 1
    for (int sweep = 0; sweep < eigh_sweeps(N); ++sweep)
#pragma unroll 1
        for (int p = 0; p < N - 1; ++p)
#pragma unroll 1
            for (int q = p + 1; q < N; ++q) {
                const T app = s[p][p], aqq = s[q][q], apq = s[p][q];
                if (!(math::abs(apq) <= (eps * math::sqrt(math::abs(app * aqq))))) {
                    const T theta = (aqq - app) / (T(2) * apq);
                    const T sg = (theta < zero) ? T(-1) : one;
                    const T tn = sg / (math::abs(theta) + math::sqrt((theta * theta) + one));
                    const T cs = one / math::sqrt((tn * tn) + one);
                    const T sn = tn * cs;
                    s[p][p] = app - (tn * apq);
                    s[q][q] = aqq + (tn * apq);
                    s[p][q] = zero;
                    s[q][p] = zero;
#pragma unroll 1
                    for (int k = 0; k < N; ++k) {
                        if ((k != p) && (k != q)) {
                            const T akp = s[k][p], akq = s[k][q];
                            const T np = (cs * akp) - (sn * akq);
                            const T nq = (sn * akp) + (cs * akq);
                            s[k][p] = np;
                            s[p][k] = np;
                            s[k][q] = nq;
                            s[q][k] = nq;
                        }
                        if (vectors) {
                            const T vp = f.v[k * N + p], vq = f.v[k * N + q];
                            f.v[k * N + p] = (cs * vp) - (sn * vq);
                            f.v[k * N + q] = (sn * vp) + (cs * vq);
                        }
                    }
                }
            }
    T off2 = zero;
#pragma unroll 1
    for (int i = 0; i < N; ++i) {
        f.w[i] = s[i][i];
#pragma unroll 1
        for (int j = 0; j < N; ++j)
            if (j != i) off2 = off2 + (s[i][j] * s[i][j]);
    }
    const T tol = static_cast<T>(N) * eps;
    if (!(off2 <= ((tol * tol) * fro2))) f.info = 1;
#pragma unroll 1
    for (int i = 0; i < N - 1; ++i) {
        int lo = i;
#pragma unroll 1
        for (int j = i + 1; j < N; ++j)
            if (f.w[j] < f.w[lo]) lo = j;
        if (lo != i) {
            const T tw = f.w[i];
            f.w[i] = f.w[lo];
            f.w[lo] = tw;
#pragma unroll 1
            for (int k = 0; k < N; ++k) {
                const T tv = f.v[k * N + i];
                f.v[k * N + i] = f.v[k * N + lo];
                f.v[k * N + lo] = tv;
            }
        }
    }
    if (vectors) {
#pragma unroll 1
        for (int j = 0; j < N; ++j) {
            int big = 0;
#pragma unroll 1
            for (int k = 1; k < N; ++k)
                if (math::abs(f.v[k * N + j]) > math::abs(f.v[big * N + j])) big = k;
            if (f.v[big * N + j] < zero)
#pragma unroll 1
                for (int k = 0; k < N; ++k) f.v[k * N + j] = -f.v[k * N + j];
        }
    }
    const T gap = tol * math::sqrt(fro2);
    bool tight = false;
#pragma unroll 1
    for (int i = 0; i < N - 1; ++i)
        if (!((f.w[i + 1] - f.w[i]) > gap)) tight = true;
    if (tight) f.info = f.info + 2;
}
}  // namespace detail

template <int N, class T, class A> HK_FI void eigh(Eigh<T, N>& f, const A& a) {
    detail::eigh_into<N, T>(f, a, true);
}

// The eigenvalues only (V is not accumulated; w and info as eigh's).
template <int N, class T, class A> HK_FI void eighValues(EighValues<T, N>& f, const A& a) {
    detail::eigh_into<N, T>(f, a, false);
}

}  // namespace linalg
}  // namespace hk
