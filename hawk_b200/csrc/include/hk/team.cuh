// hawk_b200 device library: team-form linear algebra (one matrix per lane, a
// block of threads per matrix).
//
// A factorisation too large for one thread's registers (n above the one-thread
// cap of 32, hawk/ir/linalg.py:33-36, or any n under linalg_form="team") is
// split by the reference's front end into stages (hawk/ir/team.py): a copy
// stage stores the operands row-major into the lane's slice of runtime-owned
// scratch planes, a team stage works them in place, a reader stage reads the
// results back.  The team stage's body is the reference's text
// (hawk/emit/team.py:80-113), which spells
//
//     const Team hawk_tm = Team::here();
//     const auto hawk_f = TeamCholesky<Real, n>{hawk_a, hawk_info};
//     cholesky<n>(hawk_tm, hawk_f, hawk_a);
//     choSolve<n>(hawk_tm, hawk_f, hawk_x, hawk_x, k);     // k right-hand sides, row-major n x k
//     ...
//
// and every call is collective over the block.  The b200 team is the CTA: a
// call stages the lane's matrix (row stride n + 1, so a column walk is free of
// bank conflicts) and its right-hand sides into the block's dynamic shared
// memory when the entry was given room for them, works there and writes the
// results back; otherwise it works in place on the scratch plane (L1/L2).
//
// Bits.  Every element receives the operations of the one-thread form
// (hk/linalg.cuh, the order hawk/embedded/linalg.py:188-520 restates) in the
// same order, so the team form equals the one-thread form bit for bit and no
// result depends on the team size:
//  * Cholesky, right-looking: after column k is final, every trailing entry
//    (i, j) subtracts l_ik * l_jk -- the same ascending-k chain of subtractions
//    the one-thread form's dot product applies, from the same symmetrised start
//    0.5 a_ij + 0.5 a_ji; a failed factor (info > 0) is all zeros;
//  * LU, Crout: column j's running sums acc_i = sum_{k < min(i, j)} a_ik u_kj
//    start at 0 and add in ascending k (one barrier per k: u_kj is a_kj - acc_k,
//    final once step k - 1 is done), then a_ij - acc_i; the pivot is the first
//    row of largest magnitude (a NaN diagonal keeps row j); the pivot value
//    travels with the reduction so no thread reads a row being swapped;
//  * forward sweeps run column-oriented (each x_i subtracts l_ij x_j as x_j
//    becomes final, ascending j, then divides); backward sweeps keep the
//    one-thread form's ascending-j dot product per row, so they run one thread
//    per right-hand-side column.
#pragma once
#include "base.cuh"
#include "math.cuh"
#include "stage.cuh"

namespace hk {
namespace linalg {
namespace team {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)

// The reduction scratch at the head of the dynamic shared memory: one slot per
// warp (key, value, index) for the pivot search.
constexpr unsigned kScratchBytes = 1024u;

HK_FI unsigned char* dynamic_smem() {
    extern __shared__ __align__(16) unsigned char hk_team_dyn[];
    return hk_team_dyn;
}

HK_FI unsigned dynamic_smem_bytes() {
    unsigned r;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
    return r;
}

HK_HD constexpr unsigned round16(unsigned long long b) { return static_cast<unsigned>((b + 15ull) & ~15ull); }

// Bytes of dynamic shared memory a call on an n x n matrix with k right-hand
// sides stages into: scratch, the LU running sums, the matrix (row stride
// n + 1) and the right-hand sides.  The build gives a team entry the largest of
// its calls' needs when that fits, else only the first two parts.
template <class T> HK_HD constexpr unsigned staged_bytes(int n, int k) {
    return kScratchBytes + round16(sizeof(T) * n) + round16(sizeof(T) * n * (n + 1)) + round16(sizeof(T) * n * k);
}
template <class T> HK_HD constexpr unsigned base_bytes(int n) { return kScratchBytes + round16(sizeof(T) * n); }

// The error bit a team call sets in the unit's hk_error_flags when its entry
// was launched with less dynamic shared memory than the call's scratch needs
// (the call then writes nothing but info = -1).
constexpr unsigned kErrTeamSmem = 8u;

struct Team {
    int rank;
    int size;
    static HK_FI Team here() { return Team{static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x)}; }
    HK_FI void sync() const { __syncthreads(); }
};

template <class T, int N> struct TeamCholesky {
    T* a;
    std::int32_t* info;
};

template <class T, int N> struct TeamLu {
    T* a;
    std::int32_t* piv;
    std::int32_t* info;
};

namespace detail {

// A row-major matrix with row stride ld, in shared or global memory.
template <class T> struct Mat {
    T* p;
    int ld;
    HK_FI T& operator()(int i, int j) const { return p[static_cast<long long>(i) * ld + j]; }
};

template <class T> HK_FI T* acc_of(int) { return reinterpret_cast<T*>(dynamic_smem() + kScratchBytes); }

// The working copy of a call: the matrix (staged or the scratch plane itself)
// and the right-hand sides (staged or in place).
template <class T, int N> struct Work {
    Mat<T> m;
    T* x;
    bool staged;
};

template <class T, int N> HK_FI Work<T, N> work(T* a, T* x, int k) {
    const bool staged = dynamic_smem_bytes() >= staged_bytes<T>(N, k);
    if (!staged) return Work<T, N>{Mat<T>{a, N}, x, false};
    unsigned char* base = dynamic_smem() + kScratchBytes + round16(sizeof(T) * N);
    T* m = reinterpret_cast<T*>(base);
    T* xs = reinterpret_cast<T*>(base + round16(sizeof(T) * N * (N + 1)));
    return Work<T, N>{Mat<T>{m, N + 1}, xs, true};
}

// matrix: plane (stride N) -> working copy, then a barrier
template <class T, int N> HK_FI void load_matrix(const Team& tm, const Work<T, N>& w, const T* a) {
    if (w.staged)
        for (int e = tm.rank; e < N * N; e += tm.size) w.m(e / N, e % N) = a[e];
    tm.sync();
}

template <class T, int N> HK_FI void load_rhs(const Team& tm, const Work<T, N>& w, const T* x, int k) {
    if (w.staged)
        for (int e = tm.rank; e < N * k; e += tm.size) w.x[e] = x[e];
    tm.sync();
}

template <class T, int N> HK_FI void store_rhs(const Team& tm, const Work<T, N>& w, T* x, int k) {
    if (w.staged)
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = w.x[e];
    tm.sync();
}

template <class T, int N> HK_FI void zero_rhs(const Team& tm, T* x, int k) {
    for (int e = tm.rank; e < N * k; e += tm.size) x[e] = T(0);
    tm.sync();
}

// Row i and column j of entry e of the lower triangle (diagonal included) of
// an m x m matrix, e in [0, m (m + 1) / 2), rows in ascending order.
HK_FI void tri_index(int e, int* i, int* j) {
    int r = static_cast<int>((sqrtf(8.0f * static_cast<float>(e) + 1.0f) - 1.0f) * 0.5f);
    while (r * (r + 1) / 2 > e) --r;
    while ((r + 1) * (r + 2) / 2 <= e) ++r;
    *i = r;
    *j = e - r * (r + 1) / 2;
}

// Forward sweep, column-oriented: for j ascending, x_j is final (divided by
// d(j) when `div`), then every row i > j subtracts e(i, j) * x_j.  Row i's
// subtractions come in ascending j, as the one-thread dot product makes them;
// the division of row j + 1 is done by the thread that applies its last
// subtraction, so one barrier per step.
template <class T, int N, bool DIV, class E, class D>
HK_FI void forward(const Team& tm, T* x, int k, E entry, D diag) {
    if (DIV)
        for (int c = tm.rank; c < k; c += tm.size) x[c] = x[c] / diag(0);
    tm.sync();
    for (int j = 0; j + 1 < N; ++j) {
        const int rows = N - 1 - j;
        for (int e = tm.rank; e < rows * k; e += tm.size) {
            const int i = j + 1 + e / k;
            const int c = e % k;
            T v = x[i * k + c] - (entry(i, j) * x[j * k + c]);
            if (DIV && i == j + 1) v = v / diag(i);
            x[i * k + c] = v;
        }
        tm.sync();
    }
}

// Backward sweep: for i descending, acc = x_i; acc -= e(i, j) * x_j over
// j = i + 1 .. N - 1 ascending; x_i = acc (/ d(i) when `div`).  The one-thread
// form's order, one thread per right-hand-side column.
template <class T, int N, bool DIV, class E, class D>
HK_FI void backward(const Team& tm, T* x, int k, E entry, D diag) {
    for (int c = tm.rank; c < k; c += tm.size) {
        for (int r = 0; r < N; ++r) {
            const int i = N - 1 - r;
            T acc = x[i * k + c];
            for (int j = i + 1; j < N; ++j) acc = acc - (entry(i, j) * x[j * k + c]);
            x[i * k + c] = DIV ? acc / diag(i) : acc;
        }
    }
    tm.sync();
}

// The row exchanges of a pivot vector on the right-hand sides, in step order
// or undone in reverse, one thread per column.
template <class T, int N> HK_FI void swaps(const Team& tm, T* x, int k, const std::int32_t* piv, bool ascending) {
    for (int c = tm.rank; c < k; c += tm.size) {
        for (int s = 0; s < N; ++s) {
            const int r = ascending ? s : N - 1 - s;
            const int p = piv[r];
            if (p != r) {
                const T t = x[r * k + c];
                x[r * k + c] = x[p * k + c];
                x[p * k + c] = t;
            }
        }
    }
    tm.sync();
}

}  // namespace detail

// ------------------------------------------------------------------ Cholesky

// L L^T = sym(A) in place on `a` (row-major n x n): the lower triangle holds L,
// the upper zeros; info = first failing column (1-based), and then `a` is all
// zeros (what the one-thread form's factor reads as).
template <int N, class T>
HK_FI void cholesky(const Team& tm, const TeamCholesky<T, N>& f, T* a) {
    const detail::Work<T, N> w = detail::work<T, N>(a, nullptr, 0);
    // the symmetrised lower triangle: (0.5 a_ij) + (0.5 a_ji); the reads of the
    // upper triangle are not overwritten by this pass
    for (int e = tm.rank; e < N * N; e += tm.size) {
        const int i = e / N, j = e % N;
        if (j <= i) w.m(i, j) = (T(0.5) * a[i * N + j]) + (T(0.5) * a[j * N + i]);
    }
    tm.sync();
    int info = 0;
    for (int k = 0; k < N; ++k) {
        const T d = w.m(k, k);
        if (!(d > T(0))) {
            info = k + 1;
            break;
        }
        const T lkk = math::sqrt(d);
        for (int i = k + 1 + tm.rank; i < N; i += tm.size) w.m(i, k) = w.m(i, k) / lkk;
        tm.sync();
        if (tm.rank == 0) w.m(k, k) = lkk;
        const int m = N - 1 - k;
        const int tri = m * (m + 1) / 2;
        for (int e = tm.rank; e < tri; e += tm.size) {
            int r, c;
            detail::tri_index(e, &r, &c);
            const int i = k + 1 + r, j = k + 1 + c;
            w.m(i, j) = w.m(i, j) - (w.m(i, k) * w.m(j, k));
        }
        tm.sync();
    }
    for (int e = tm.rank; e < N * N; e += tm.size) {
        const int i = e / N, j = e % N;
        a[e] = (info == 0 && j <= i) ? w.m(i, j) : T(0);
    }
    if (tm.rank == 0) *f.info = info;
    tm.sync();
}

// The lower triangle of `a` taken as the factor: info = first column whose
// diagonal entry is not positive and finite; the upper triangle is zeroed, and
// a failed factor is all zeros.
template <int N, class T>
HK_FI void choleskyFrom(const Team& tm, const TeamCholesky<T, N>& f, T* a) {
    int info = 0;
    for (int j = 0; j < N; ++j) {
        const T d = a[j * N + j];
        if ((d <= T(0)) || !math::isfinite(d)) {
            info = j + 1;
            break;
        }
    }
    tm.sync();                  // every thread has read the diagonal before it changes
    for (int e = tm.rank; e < N * N; e += tm.size) {
        const int i = e / N, j = e % N;
        if (info != 0 || j > i) a[e] = T(0);
    }
    if (tm.rank == 0) *f.info = info;
    tm.sync();
}

// x = A^{-1} b from the factor, k right-hand sides (row-major n x k), in place
// when b == x: forward sweep on L, backward on L^T; zeros for a failed factor.
template <int N, class T>
HK_FI void choSolve(const Team& tm, const TeamCholesky<T, N>& f, const T* b, T* x, int k) {
    if (*f.info != 0) {
        detail::zero_rhs<T, N>(tm, x, k);
        return;
    }
    if (b != x) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = b[e];
        tm.sync();
    }
    const detail::Work<T, N> w = detail::work<T, N>(f.a, x, k);
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const detail::Mat<T> l = w.m;
    detail::forward<T, N, true>(tm, w.x, k, [&](int i, int j) { return l(i, j); }, [&](int i) { return l(i, i); });
    detail::backward<T, N, true>(tm, w.x, k, [&](int i, int j) { return l(j, i); }, [&](int i) { return l(i, i); });
    detail::store_rhs<T, N>(tm, w, x, k);
}

// L y = b (forward, on the factor's L) and L^T y = b (backward).
template <int N, class T>
HK_FI void triLower(const Team& tm, const TeamCholesky<T, N>& f, const T* b, T* x, int k) {
    if (b != x) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = b[e];
        tm.sync();
    }
    const detail::Work<T, N> w = detail::work<T, N>(f.a, x, k);
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const detail::Mat<T> l = w.m;
    detail::forward<T, N, true>(tm, w.x, k, [&](int i, int j) { return l(i, j); }, [&](int i) { return l(i, i); });
    detail::store_rhs<T, N>(tm, w, x, k);
}

template <int N, class T>
HK_FI void triUpperT(const Team& tm, const TeamCholesky<T, N>& f, const T* b, T* x, int k) {
    if (b != x) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = b[e];
        tm.sync();
    }
    const detail::Work<T, N> w = detail::work<T, N>(f.a, x, k);
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const detail::Mat<T> l = w.m;
    detail::backward<T, N, true>(tm, w.x, k, [&](int i, int j) { return l(j, i); }, [&](int i) { return l(i, i); });
    detail::store_rhs<T, N>(tm, w, x, k);
}

// ------------------------------------------------------------------------ LU

// P A = L U in place (Crout, column by column); piv[j] = the row exchanged
// with row j at step j; info = first zero pivot column (1-based).
template <int N, class T>
HK_FI void lu(const Team& tm, const TeamLu<T, N>& f, T* a) {
    if (dynamic_smem_bytes() < base_bytes<T>(N)) {
        if (tm.rank == 0) {
            stage::fail(kErrTeamSmem);
            *f.info = -1;
        }
        tm.sync();
        return;
    }
    const detail::Work<T, N> w = detail::work<T, N>(a, nullptr, 0);
    detail::load_matrix<T, N>(tm, w, a);
    T* acc = detail::acc_of<T>(N);
    T* red_key = reinterpret_cast<T*>(dynamic_smem());
    T* red_val = red_key + 32;
    int* red_idx = reinterpret_cast<int*>(red_val + 32);
    for (int i = tm.rank; i < N; i += tm.size) acc[i] = T(0);
    tm.sync();
    int info = 0;
    const int lane = tm.rank & 31, warp = tm.rank >> 5, warps = (tm.size + 31) >> 5;
    for (int j = 0; j < N; ++j) {
        // running sums: acc_i += a_ik * u_kj once u_kj = a_kj - acc_k is final
        for (int k = 0; k + 1 < N && k < j; ++k) {
            const T ukj = w.m(k, j) - acc[k];
            for (int i = k + 1 + tm.rank; i < N; i += tm.size) acc[i] = acc[i] + (w.m(i, k) * ukj);
            tm.sync();
        }
        for (int i = tm.rank; i < N; i += tm.size) {
            w.m(i, j) = w.m(i, j) - acc[i];
            acc[i] = T(0);
        }
        tm.sync();
        // pivot: the first row of largest magnitude at or below the diagonal
        const T ajj = w.m(j, j);
        T bkey = T(-2), bval = T(0);
        int bidx = N;
        for (int i = j + tm.rank; i < N; i += tm.size) {
            const T v = w.m(i, j);
            const T mag = math::abs(v);
            const T key = math::isnan(mag) ? T(-1) : mag;
            if (key > bkey) {
                bkey = key;
                bval = v;
                bidx = i;
            }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const T ok = __shfl_down_sync(0xffffffffu, bkey, off);
            const T ov = __shfl_down_sync(0xffffffffu, bval, off);
            const int oi = __shfl_down_sync(0xffffffffu, bidx, off);
            if (lane + off < 32 && (ok > bkey || (ok == bkey && oi < bidx))) {
                bkey = ok;
                bval = ov;
                bidx = oi;
            }
        }
        if (lane == 0) {
            red_key[warp] = bkey;
            red_val[warp] = bval;
            red_idx[warp] = bidx;
        }
        tm.sync();
        T pkey = red_key[0], pj = red_val[0];
        int p = red_idx[0];
        for (int q = 1; q < warps; ++q) {
            const T ok = red_key[q];
            const int oi = red_idx[q];
            if (ok > pkey || (ok == pkey && oi < p)) {
                pkey = ok;
                pj = red_val[q];
                p = oi;
            }
        }
        if (math::isnan(math::abs(ajj))) {
            p = j;
            pj = ajj;
        }
        if (tm.rank == 0) f.piv[j] = p;
        if (pj != T(0)) {
            const T rcp = T(1) / pj;
            if (p != j)
                for (int c = tm.rank; c < N; c += tm.size) {
                    if (c == j) continue;
                    const T t = w.m(j, c);
                    w.m(j, c) = w.m(p, c);
                    w.m(p, c) = t;
                }
            for (int i = j + 1 + tm.rank; i < N; i += tm.size)
                if (i != p) w.m(i, j) = w.m(i, j) * rcp;
            if (tm.rank == 0 && p != j) {
                w.m(p, j) = ajj * rcp;
                w.m(j, j) = pj;
            }
        } else if (info == 0) {
            info = j + 1;
        }
        tm.sync();
    }
    if (w.staged)
        for (int e = tm.rank; e < N * N; e += tm.size) a[e] = w.m(e / N, e % N);
    if (tm.rank == 0) *f.info = info;
    tm.sync();
}

// x = A^{-1} b from the factor: the exchanges in step order, the unit-lower
// forward sweep, the backward sweep on U; zeros for a failed factor.
template <int N, class T>
HK_FI void luSolve(const Team& tm, const TeamLu<T, N>& f, const T* b, T* x, int k) {
    if (*f.info != 0) {
        detail::zero_rhs<T, N>(tm, x, k);
        return;
    }
    if (b != x) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = b[e];
        tm.sync();
    }
    const detail::Work<T, N> w = detail::work<T, N>(f.a, x, k);
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const detail::Mat<T> u = w.m;
    detail::swaps<T, N>(tm, w.x, k, f.piv, true);
    detail::forward<T, N, false>(tm, w.x, k, [&](int i, int j) { return u(i, j); }, [&](int) { return T(1); });
    detail::backward<T, N, true>(tm, w.x, k, [&](int i, int j) { return u(i, j); }, [&](int i) { return u(i, i); });
    detail::store_rhs<T, N>(tm, w, x, k);
}

// x = A^{-T} b: U^T forward (with U's diagonal), L^T backward (unit), then the
// exchanges undone in reverse; zeros for a failed factor.
template <int N, class T>
HK_FI void luSolveT(const Team& tm, const TeamLu<T, N>& f, const T* b, T* x, int k) {
    if (*f.info != 0) {
        detail::zero_rhs<T, N>(tm, x, k);
        return;
    }
    if (b != x) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = b[e];
        tm.sync();
    }
    const detail::Work<T, N> w = detail::work<T, N>(f.a, x, k);
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const detail::Mat<T> u = w.m;
    detail::forward<T, N, true>(tm, w.x, k, [&](int i, int j) { return u(j, i); }, [&](int i) { return u(i, i); });
    detail::backward<T, N, false>(tm, w.x, k, [&](int i, int j) { return u(j, i); }, [&](int) { return T(1); });
    detail::swaps<T, N>(tm, w.x, k, f.piv, false);
    detail::store_rhs<T, N>(tm, w, x, k);
}

// A^{-1} into x (n x n): the solve of the identity.
template <int N, class T>
HK_FI void luInverse(const Team& tm, const TeamLu<T, N>& f, T* x) {
    for (int e = tm.rank; e < N * N; e += tm.size) x[e] = (e / N == e % N) ? T(1) : T(0);
    tm.sync();
    luSolve<N>(tm, f, x, x, N);
}

// det(A): the product of U's diagonal, negated per exchange as it is met
// (hawk/embedded/linalg.py:402-418); 0 for a failed factor.  One thread.
template <int N, class T>
HK_FI T luDet(const TeamLu<T, N>& f) {
    T d = T(0);
    if (*f.info == 0) {
        d = T(1);
        for (int k = 0; k < N; ++k) {
            d = d * f.a[k * N + k];
            if (f.piv[k] != k) d = -d;
        }
    }
    return d;
}

#endif  // __CUDACC__

}  // namespace team
}  // namespace linalg
}  // namespace hk
