// hawk_b200 device library: team-form linear algebra (one matrix per lane, a
// team of threads -- one warp -- per matrix).
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
// and every call is collective over the team.  The b200 team is one warp (a
// block of the entry serves one lane per warp, so many lanes are in flight
// per SM and a call's barriers are the warp's): a call stages the lane's matrix (row stride n + 1, so a column walk is free of
// bank conflicts) and its right-hand sides into the block's dynamic shared
// memory when the entry was given room for them, works there and writes the
// results back; otherwise it works in place on the scratch plane (L1/L2).  A
// factor left staged by its factorisation is reused by the solves after it
// (a tag holds the scratch-plane address the staged copy stands for).
//
// Bits.  Every element receives the operations of the one-thread form
// (hk/linalg.cuh, the order hawk/embedded/linalg.py:188-520 restates) in the
// same order, so the team form equals the one-thread form bit for bit and no
// result depends on the team size:
//  * Cholesky, column by column: row i >= j of column j starts from the
//    symmetrised 0.5 a_ij + 0.5 a_ji and subtracts l_ik * l_jk in ascending k
//    in a register (the one-thread form's dot product, lanes over rows), then
//    divides by l_jj; a failed factor (info > 0) is all zeros;
//  * LU, Crout, by the team's first warp: column j's running sums
//    acc_i = sum_{k < min(i, j)} a_ik u_kj start at 0 and add in ascending k
//    (u_kj = a_kj - acc_k is final once k - 1 is done), then a_ij - acc_i; the
//    pivot is the first row of largest magnitude (a NaN diagonal keeps row j),
//    its value travels with the warp reduction;
//  * forward sweeps run column-oriented (each x_i subtracts l_ij x_j as x_j
//    becomes final, ascending j, then divides); backward sweeps keep the
//    one-thread form's ascending-j dot product per row, so they run one thread
//    per right-hand-side column.
#pragma once
#include "base.cuh"
#include "math.cuh"

namespace hk {
namespace linalg {
namespace team {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)

}  // namespace team
}  // namespace linalg
}  // namespace hk
extern "C" __device__ unsigned int hk_error_flags;     // the unit's error word (HK_SELF_CHECK_EXPORTS defines it)
namespace hk {
namespace linalg {
namespace team {

// The head of a team entry's dynamic shared memory: the staged-factor tag
// (below) in its last 16 bytes; the staged matrix and right-hand sides follow.
constexpr unsigned kScratchBytes = 128u;

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

// Bytes of dynamic shared memory a team's calls on an n x n matrix with k
// right-hand sides use: the head and the products row of the backward sweeps
// (inplace_bytes), plus, to stage, the matrix (row stride n + 1) and the
// right-hand sides.  The build gives each team of an entry the largest staged
// need of its calls when that fits, else the in-place need.
template <class T> HK_HD constexpr unsigned inplace_bytes(int n) { return kScratchBytes + round16(sizeof(T) * n); }
template <class T> HK_HD constexpr unsigned staged_bytes(int n, int k) {
    return inplace_bytes<T>(n) + round16(sizeof(T) * n * (n + 1)) + round16(sizeof(T) * n * k);
}
// The Cholesky family reads and writes only the lower triangle: staged, it is
// packed by rows (n (n + 1) / 2 entries), half the full copy, so twice as many
// teams fit an SM.
template <class T> HK_HD constexpr unsigned staged_lower_bytes(int n, int k) {
    return inplace_bytes<T>(n) + round16(sizeof(T) * n * (n + 1) / 2) + round16(sizeof(T) * n * k);
}

// The team of a lane: one warp.  A team entry's block holds several warps,
// each on a lane of its own (the team frame), so a call's barrier is the
// warp's and many lanes are in flight per SM; the block's dynamic shared
// memory is split evenly between its warps, each staging into its own part.
struct Team {
    int rank;                   // the thread's place in the team (its lane in the warp)
    int size;                   // 32
    unsigned char* smem;        // this team's part of the block's dynamic shared memory
    unsigned bytes;             // its size
    static HK_FI Team here() {
        const unsigned warps = blockDim.x >> 5;
        const unsigned part = (dynamic_smem_bytes() / (warps ? warps : 1u)) & ~15u;
        return Team{static_cast<int>(threadIdx.x & 31u), 32, dynamic_smem() + (threadIdx.x >> 5) * part, part};
    }
    HK_FI void sync() const { __syncwarp(); }
};

// The staged-factor tag at the end of a team's head: the scratch-plane
// address of the matrix its staged copy holds (a factor a solve can reuse).
constexpr unsigned kTagOffset = kScratchBytes - 16u;
HK_FI const void* volatile* tag_slot(const Team& tm) {
    return reinterpret_cast<const void* volatile*>(tm.smem + kTagOffset);
}

// At the start of a team entry: no staged copy is held yet.  Every thread of
// the block calls it.
HK_FI void begin_entry() {
    const Team tm = Team::here();
    if (tm.bytes >= kScratchBytes && tm.rank == 0) *tag_slot(tm) = nullptr;
    __syncwarp();
}

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

// A lower triangle packed by rows in shared memory has entry (i, j), j <= i,
// at i (i + 1) / 2 + j.  The rows' offsets are the triangular numbers, which
// are distinct modulo 32 over any 32 consecutive rows, so a column walk across
// the lanes is free of bank conflicts.  EitherMat is a row-major matrix
// (ld > 0) or, with ld == 0, such a triangle: one accessor for a call that may
// run staged or in place keeps one code path (and one register budget).
template <class T> struct EitherMat {
    T* p;
    int ld;
    HK_FI T& operator()(int i, int j) const {
        const long long row = ld ? static_cast<long long>(i) * ld : static_cast<long long>((i * (i + 1)) >> 1);
        return p[row + j];
    }
};

// The packed lower triangle's select-free accessor, for a unit whose team
// stage always stages it (HK_TEAM_LOWER_STAGED == 1).
template <class T> struct Tri {
    T* p;
    int ld;                     // unused: the layout is the triangle's
    HK_FI T& operator()(int i, int j) const { return p[((i * (i + 1)) >> 1) + j]; }
};

// The working copy of a call: the matrix (staged or the scratch plane itself)
// and the right-hand sides (staged or in place); `lower` when the staged copy
// is a packed lower triangle.
template <class T, int N, class M = Mat<T>> struct Work {
    M m;
    T* x;
    bool staged;
    bool lower;
};

// How a unit's Cholesky-family calls (which read and write only the lower
// triangle) hold their matrix, set by the build before the library is
// included: 1, the team stage's shared memory holds every call's packed
// triangle (the accessor is Tri); 0, no call stages (the plane, in place);
// undefined, decided per call by the team's shared memory (EitherMat).
#if defined(HK_TEAM_LOWER_STAGED) && HK_TEAM_LOWER_STAGED == 1
template <class T> using LowerMat = Tri<T>;
#elif defined(HK_TEAM_LOWER_STAGED) && HK_TEAM_LOWER_STAGED == 0
template <class T> using LowerMat = Mat<T>;
#else
template <class T> using LowerMat = EitherMat<T>;
#endif

// Error bit of the unit's hk_error_flags word (hk/stage.cuh holds the others):
// a team's shared memory did not hold the packed triangle its unit was built
// to stage; the call did nothing.
constexpr unsigned kErrTeamSmem = 8u;

// The working copy of a Cholesky-family call: the packed triangle and the
// right-hand sides staged, or the plane itself and the right-hand sides in
// place, as the unit was built (above).  `ok` is false when a unit built to
// stage finds too little shared memory (never, by the build's sizing).
template <class T, int N> HK_FI Work<T, N, LowerMat<T>> work_lower(const Team& tm, T* a, T* x, int k, bool* ok) {
    *ok = true;
    const bool fits = tm.bytes >= staged_lower_bytes<T>(N, k);
    unsigned char* base = tm.smem + inplace_bytes<T>(N);
    T* tri = reinterpret_cast<T*>(base);
    T* xs = reinterpret_cast<T*>(base + round16(sizeof(T) * N * (N + 1) / 2));
#if defined(HK_TEAM_LOWER_STAGED) && HK_TEAM_LOWER_STAGED == 1
    if (!fits) {
        *ok = false;
        if (tm.rank == 0) atomicOr(&hk_error_flags, kErrTeamSmem);
    }
    return Work<T, N, LowerMat<T>>{LowerMat<T>{tri, 0}, xs, true, true};
#elif defined(HK_TEAM_LOWER_STAGED) && HK_TEAM_LOWER_STAGED == 0
    (void)fits, (void)tri, (void)xs;
    return Work<T, N, LowerMat<T>>{LowerMat<T>{a, N}, x, false, false};
#else
    if (!fits) return Work<T, N, LowerMat<T>>{LowerMat<T>{a, N}, x, false, false};
    return Work<T, N, LowerMat<T>>{LowerMat<T>{tri, 0}, xs, true, true};
#endif
}

// The staged-factor tag of plane address a for a working copy: a packed copy
// is tagged one byte past it, so a full copy never takes a packed one for its
// own.
template <class T, int N, class M> HK_FI const void* tag_of(const Work<T, N, M>& w, const T* a) {
    return static_cast<const void*>(reinterpret_cast<const unsigned char*>(a) + (w.lower ? 1 : 0));
}

template <class T, int N> HK_FI Work<T, N> work(const Team& tm, T* a, T* x, int k) {
    const bool staged = tm.bytes >= staged_bytes<T>(N, k);
    if (!staged) return Work<T, N>{Mat<T>{a, N}, x, false, false};
    unsigned char* base = tm.smem + inplace_bytes<T>(N);
    T* m = reinterpret_cast<T*>(base);
    T* xs = reinterpret_cast<T*>(base + round16(sizeof(T) * N * (N + 1)));
    return Work<T, N>{Mat<T>{m, N + 1}, xs, true, false};
}

// An elementwise pass over e in [0, count) by the team, U entries of a thread
// at a time with every load of the batch issued before any store (the
// compiler cannot tell the two sides apart, and in place they may be the same
// array): value(e) is read, store(e, v) written.
template <int U, class V, class S> HK_FI void batched(const Team& tm, int count, V value, S store) {
    for (int e0 = tm.rank; e0 < count; e0 += U * tm.size) {
        decltype(value(0)) v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (e0 + u * tm.size < count) v[u] = value(e0 + u * tm.size);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (e0 + u * tm.size < count) store(e0 + u * tm.size, v[u]);
    }
}

// matrix: plane (stride N) -> working copy, then a barrier; a copy the
// staged area already holds (the factor the previous call made) is kept
template <class T, int N, class M> HK_FI void load_matrix(const Team& tm, const Work<T, N, M>& w, const T* a) {
    if (w.staged && *tag_slot(tm) != tag_of(w, a)) {
        tm.sync();              // every thread has read the tag before it changes
        batched<8>(tm, N * N, [&](int e) { return (!w.lower || e % N <= e / N) ? a[e] : T(0); },
                   [&](int e, T v) {
                       if (!w.lower || e % N <= e / N) w.m(e / N, e % N) = v;
                   });
        if (tm.rank == 0) *tag_slot(tm) = tag_of(w, a);
    }
    tm.sync();
}

// the staged area now holds the final matrix of plane address a (or nothing)
template <class T> HK_FI void set_tag(const Team& tm, const T* a) {
    if (tm.rank == 0) *tag_slot(tm) = static_cast<const void*>(a);
}

template <class T, int N, class M> HK_FI void load_rhs(const Team& tm, const Work<T, N, M>& w, const T* x, int k) {
    if (w.staged)
        for (int e = tm.rank; e < N * k; e += tm.size) w.x[e] = x[e];
    tm.sync();
}

template <class T, int N, class M> HK_FI void store_rhs(const Team& tm, const Work<T, N, M>& w, T* x, int k) {
    if (w.staged)
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = w.x[e];
    tm.sync();
}

template <class T, int N> HK_FI void zero_rhs(const Team& tm, T* x, int k) {
    for (int e = tm.rank; e < N * k; e += tm.size) x[e] = T(0);
    tm.sync();
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
// form's order: the subtractions of a row are one chain, so one thread runs
// it; the products it subtracts (independent of one another, all of final
// x_j) are made by the whole team into the products row first.
template <class T, int N, bool DIV, class E, class D>
HK_FI void backward(const Team& tm, T* x, int k, E entry, D diag) {
    if (tm.bytes >= inplace_bytes<T>(N) && k == 1) {
        T* prod = reinterpret_cast<T*>(tm.smem + kScratchBytes);
        for (int r = 0; r < N; ++r) {
            const int i = N - 1 - r;
            for (int j = i + 1 + tm.rank; j < N; j += tm.size) prod[j] = entry(i, j) * x[j];
            tm.sync();
            if (tm.rank == 0) {
                T acc = x[i];
#pragma unroll 8
                for (int j = i + 1; j < N; ++j) acc = acc - prod[j];
                x[i] = DIV ? acc / diag(i) : acc;
            }
            tm.sync();
        }
        return;
    }
    for (int c = tm.rank; c < k; c += tm.size) {
        for (int r = 0; r < N; ++r) {
            const int i = N - 1 - r;
            T acc = x[i * k + c];
            // the products are independent of the chain: unrolled so their loads
            // are in flight while the subtractions run in order
#pragma unroll 8
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
    bool ok = true;
    const auto w = detail::work_lower<T, N>(tm, a, nullptr, 0, &ok);
    if (!ok) return;
    if (w.staged) {
        tm.sync();              // every thread has read the tag before it changes
        detail::set_tag(tm, static_cast<const T*>(nullptr));
    }
    // the symmetrised lower triangle: (0.5 a_ij) + (0.5 a_ji); the reads of the
    // upper triangle are not overwritten by this pass
    detail::batched<8>(tm, N * N,
                       [&](int e) {
                           const int i = e / N, j = e % N;
                           return j <= i ? (T(0.5) * a[i * N + j]) + (T(0.5) * a[j * N + i]) : T(0);
                       },
                       [&](int e, T v) {
                           if (e % N <= e / N) w.m(e / N, e % N) = v;
                       });
    tm.sync();
    // Column by column, the one-thread form's own order: row i >= j of column
    // j starts from its symmetrised entry and subtracts l_ik * l_jk for
    // k = 0 .. j - 1 in a register (the diagonal's terms are l_jk * l_jk),
    // then divides by l_jj = sqrt of the diagonal's result.  Rows are the
    // lanes' (row i on lane i % 32); one warp barrier per column.
    constexpr int R = (N + 31) / 32;
    constexpr unsigned kAll = 0xffffffffu;
    const int lane = tm.rank;
    int info = 0;
    for (int j = 0; j < N; ++j) {
        T acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = lane + 32 * r;
            acc[r] = (i >= j && i < N) ? w.m(i, j) : T(0);
        }
        // four k at a time: the loads and products of a group are issued
        // ahead of its chain of subtractions (which keeps ascending k)
        int k = 0;
        for (; k + 4 <= j; k += 4) {
            T lj[4], p[R][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) lj[u] = w.m(j, k + u);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = lane + 32 * r;
                const int ii = (i >= j && i < N) ? i : j;
#pragma unroll
                for (int u = 0; u < 4; ++u) p[r][u] = w.m(ii, k + u) * lj[u];
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = lane + 32 * r;
                if (i >= j && i < N)
#pragma unroll
                    for (int u = 0; u < 4; ++u) acc[r] = acc[r] - p[r][u];
            }
        }
        for (; k < j; ++k) {
            const T ljk = w.m(j, k);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = lane + 32 * r;
                if (i >= j && i < N) acc[r] = acc[r] - (w.m(i, k) * ljk);
            }
        }
        T mine = T(0);
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (r == (j >> 5)) mine = acc[r];
        const T d = __shfl_sync(kAll, mine, j & 31);
        if (!(d > T(0))) {
            info = j + 1;
            break;
        }
        const T ljj = math::sqrt(d);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = lane + 32 * r;
            if (i > j && i < N) w.m(i, j) = acc[r] / ljj;
        }
        if (lane == (j & 31)) w.m(j, j) = ljj;
        tm.sync();
    }
    tm.sync();
    detail::batched<8>(tm, N * N,
                       [&](int e) {
                           const int i = e / N, j = e % N;
                           return (info == 0 && j <= i) ? w.m(i, j) : T(0);
                       },
                       [&](int e, T v) { a[e] = v; });
    if (tm.rank == 0) *f.info = info;
    if (w.staged && info == 0) detail::set_tag(tm, detail::tag_of(w, a));
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
    tm.sync();                  // every thread has read the diagonal (and the tag) before they change
    for (int e = tm.rank; e < N * N; e += tm.size) {
        const int i = e / N, j = e % N;
        if (info != 0 || j > i) a[e] = T(0);
    }
    if (tm.rank == 0) *f.info = info;
    if (tm.bytes >= kScratchBytes) detail::set_tag(tm, static_cast<const T*>(nullptr));
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
    bool ok = true;
    const auto w = detail::work_lower<T, N>(tm, f.a, x, k, &ok);
    if (!ok) return;
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const auto l = w.m;
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
    bool ok = true;
    const auto w = detail::work_lower<T, N>(tm, f.a, x, k, &ok);
    if (!ok) return;
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const auto l = w.m;
    detail::forward<T, N, true>(tm, w.x, k, [&](int i, int j) { return l(i, j); }, [&](int i) { return l(i, i); });
    detail::store_rhs<T, N>(tm, w, x, k);
}

template <int N, class T>
HK_FI void triUpperT(const Team& tm, const TeamCholesky<T, N>& f, const T* b, T* x, int k) {
    if (b != x) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = b[e];
        tm.sync();
    }
    bool ok = true;
    const auto w = detail::work_lower<T, N>(tm, f.a, x, k, &ok);
    if (!ok) return;
    detail::load_matrix<T, N>(tm, w, f.a);
    detail::load_rhs<T, N>(tm, w, x, k);
    const auto l = w.m;
    detail::backward<T, N, true>(tm, w.x, k, [&](int i, int j) { return l(j, i); }, [&](int i) { return l(i, i); });
    detail::store_rhs<T, N>(tm, w, x, k);
}

// ------------------------------------------------------------------------ LU

// P A = L U in place (Crout, column by column); piv[j] = the row exchanged
// with row j at step j; info = first zero pivot column (1-based).  Row i's
// running sum lives in the registers of lane i % 32, u_kj goes from the lane
// owning row k to the others by a shuffle, the pivot is a warp reduction.
template <int N, class T>
HK_FI void lu(const Team& tm, const TeamLu<T, N>& f, T* a) {
    const detail::Work<T, N> w = detail::work<T, N>(tm, a, nullptr, 0);
    if (w.staged) {
        tm.sync();              // every thread has read the tag before it changes
        detail::set_tag(tm, static_cast<const T*>(nullptr));
        tm.sync();
    }
    detail::load_matrix<T, N>(tm, w, a);
    constexpr int R = (N + 31) / 32;        // rows per lane
    constexpr unsigned kAll = 0xffffffffu;
    int info = 0;
    if (tm.rank < 32) {
        const int lane = tm.rank;
        for (int j = 0; j < N; ++j) {
            T acc[R], col[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = lane + 32 * r;
                acc[r] = T(0);
                col[r] = i < N ? w.m(i, j) : T(0);       // column j, held for the chain below
            }
            // Crout: acc_i = sum_{k < min(i, j)} a_ik u_kj, ascending k from 0;
            // u_kj = a_kj - acc_k is final once every k' < k was added
            for (int k = 0; k < j; ++k) {
                const int slot = k >> 5;
                T mine = T(0);
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (r == slot) mine = col[r] - acc[r];
                const T ukj = __shfl_sync(kAll, mine, k & 31);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int i = lane + 32 * r;
                    if (i > k && i < N) acc[r] = acc[r] + (w.m(i, k) * ukj);
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = lane + 32 * r;
                if (i < N) w.m(i, j) = col[r] - acc[r];
            }
            __syncwarp();
            // pivot: the first row of largest magnitude at or below the diagonal
            const T ajj = w.m(j, j);
            T bkey = T(-2), bval = T(0);
            int bidx = N;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = lane + 32 * r;
                if (i >= j && i < N) {
                    const T v = w.m(i, j);
                    const T mag = math::abs(v);
                    const T key = math::isnan(mag) ? T(-1) : mag;
                    if (key > bkey) {
                        bkey = key;
                        bval = v;
                        bidx = i;
                    }
                }
            }
            for (int off = 16; off > 0; off >>= 1) {
                const T ok = __shfl_xor_sync(kAll, bkey, off);
                const T ov = __shfl_xor_sync(kAll, bval, off);
                const int oi = __shfl_xor_sync(kAll, bidx, off);
                if (ok > bkey || (ok == bkey && oi < bidx)) {
                    bkey = ok;
                    bval = ov;
                    bidx = oi;
                }
            }
            int p = bidx;
            T pj = bval;
            if (math::isnan(math::abs(ajj))) {
                p = j;
                pj = ajj;
            }
            __syncwarp();       // every lane has read a_jj before it changes
            if (lane == 0) f.piv[j] = p;
            if (pj != T(0)) {
                const T rcp = T(1) / pj;
                if (p != j)
                    for (int c = lane; c < N; c += 32) {
                        if (c == j) continue;
                        const T t = w.m(j, c);
                        w.m(j, c) = w.m(p, c);
                        w.m(p, c) = t;
                    }
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int i = lane + 32 * r;
                    if (i > j && i < N && i != p) w.m(i, j) = w.m(i, j) * rcp;
                }
                if (lane == 0 && p != j) {
                    w.m(p, j) = ajj * rcp;
                    w.m(j, j) = pj;
                }
            } else if (info == 0) {
                info = j + 1;
            }
            __syncwarp();
        }
    }
    tm.sync();
    if (w.staged)
        detail::batched<8>(tm, N * N, [&](int e) { return w.m(e / N, e % N); }, [&](int e, T v) { a[e] = v; });
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
    const detail::Work<T, N> w = detail::work<T, N>(tm, f.a, x, k);
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
    const detail::Work<T, N> w = detail::work<T, N>(tm, f.a, x, k);
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

// ----------------------------------------------------- symmetric eigenproblem

template <class T, int N> struct TeamEigh {
    T* w;
    T* v;
    T* work;
    std::int32_t* info;
};

// w, V, info of the symmetric part of `a` (n x n, row-major): the one-thread
// form's cyclic Jacobi (hk/linalg.cuh eigh, hawk/embedded/linalg.py:302-399)
// with each rotation's row and column updates spread over the team (every k
// gets the one-thread form's operations), the rotation's own scalars made by
// every thread alike, and the epilogue (ordering, signs, status) by one thread:
// the one-thread form's bits.  The working matrix is staged in the team's
// shared memory when it fits, else kept in `work` (n^2 + 4).
template <int N, class T>
HK_FI void eigh(const Team& tm, const TeamEigh<T, N>& f, T* a) {
    const T zero = T(0), one = T(1), half = T(0.5);
    const T eps = linalg::EighEps<T>::value();
    T* s = (tm.bytes >= kScratchBytes + sizeof(T) * N * N) ? reinterpret_cast<T*>(tm.smem + kScratchBytes) : f.work;
    if (tm.bytes >= kScratchBytes) {
        tm.sync();
        detail::set_tag(tm, static_cast<const T*>(nullptr));
    }
    for (int e = tm.rank; e < N * N; e += tm.size) {
        const int i = e / N, j = e % N;
        s[e] = (j >= i) ? (half * a[i * N + j]) + (half * a[j * N + i]) : T(0);
        f.v[e] = (i == j) ? one : zero;
    }
    tm.sync();
    T fro2 = zero;
    if (N == 1) {
        if (tm.rank == 0) {
            f.w[0] = a[0];
            *f.info = 0;
        }
        tm.sync();
        return;
    }
    // the lower half mirrors the upper (what the one-thread fill copies), and
    // the Frobenius sum in the fill's order: one thread
    if (tm.rank == 0) {
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < N; ++j) {
                if (j < i) s[i * N + j] = s[j * N + i];
                fro2 = fro2 + (s[i * N + j] * s[i * N + j]);
            }
    }
    tm.sync();
    for (int sweep = 0; sweep < linalg::eigh_sweeps(N); ++sweep)
        for (int p = 0; p < N - 1; ++p)
            for (int q = p + 1; q < N; ++q) {
                const T app = s[p * N + p], aqq = s[q * N + q], apq = s[p * N + q];
                tm.sync();              // every thread has read the pivot block before it changes
                if (!(math::abs(apq) <= (eps * math::sqrt(math::abs(app * aqq))))) {
                    const T theta = (aqq - app) / (T(2) * apq);
                    const T sg = (theta < zero) ? T(-1) : one;
                    const T tn = sg / (math::abs(theta) + math::sqrt((theta * theta) + one));
                    const T cs = one / math::sqrt((tn * tn) + one);
                    const T sn = tn * cs;
                    if (tm.rank == 0) {
                        s[p * N + p] = app - (tn * apq);
                        s[q * N + q] = aqq + (tn * apq);
                        s[p * N + q] = zero;
                        s[q * N + p] = zero;
                    }
                    for (int k = tm.rank; k < N; k += tm.size) {
                        if ((k != p) && (k != q)) {
                            const T akp = s[k * N + p], akq = s[k * N + q];
                            const T np = (cs * akp) - (sn * akq);
                            const T nq = (sn * akp) + (cs * akq);
                            s[k * N + p] = np;
                            s[p * N + k] = np;
                            s[k * N + q] = nq;
                            s[q * N + k] = nq;
                        }
                        const T vp = f.v[k * N + p], vq = f.v[k * N + q];
                        f.v[k * N + p] = (cs * vp) - (sn * vq);
                        f.v[k * N + q] = (sn * vp) + (cs * vq);
                    }
                }
                tm.sync();
            }
    if (tm.rank == 0) {
        int info = 0;
        T off2 = zero;
        for (int i = 0; i < N; ++i) {
            f.w[i] = s[i * N + i];
            for (int j = 0; j < N; ++j)
                if (j != i) off2 = off2 + (s[i * N + j] * s[i * N + j]);
        }
        const T tol = static_cast<T>(N) * eps;
        if (!(off2 <= ((tol * tol) * fro2))) info = 1;
        for (int i = 0; i < N - 1; ++i) {
            int lo = i;
            for (int j = i + 1; j < N; ++j)
                if (f.w[j] < f.w[lo]) lo = j;
            if (lo != i) {
                const T tw = f.w[i];
                f.w[i] = f.w[lo];
                f.w[lo] = tw;
                for (int k = 0; k < N; ++k) {
                    const T tv = f.v[k * N + i];
                    f.v[k * N + i] = f.v[k * N + lo];
                    f.v[k * N + lo] = tv;
                }
            }
        }
        for (int j = 0; j < N; ++j) {
            int big = 0;
            for (int k = 1; k < N; ++k)
                if (math::abs(f.v[k * N + j]) > math::abs(f.v[big * N + j])) big = k;
            if (f.v[big * N + j] < zero)
                for (int k = 0; k < N; ++k) f.v[k * N + j] = -f.v[k * N + j];
        }
        const T gap = tol * math::sqrt(fro2);
        bool tight = false;
        for (int i = 0; i < N - 1; ++i)
            if (!((f.w[i + 1] - f.w[i]) > gap)) tight = true;
        *f.info = tight ? info + 2 : info;
    }
    tm.sync();
}

// ------------------------------------------------------ QR least squares

template <class T, int N> struct TeamQr {
    T* a;
    T* tau;
    T* work;
    std::int32_t* info;
};

// Householder QR of the m x n matrix `a` (row-major, m >= n) in place: for
// column j, the sum of squares of a_ij, i >= j (ascending i, one thread),
// its root `norm`, R_jj = alpha = -sign(a_jj) norm (sign(0) = +1), the
// reflector v = (a_jj - alpha, a_{j+1..m-1, j}) kept below the diagonal with
// v_0 in work[j] and tau_j = 2 / v.v; each later column c (one thread per
// column) takes d = v_0 a_jc + sum_{i>j} a_ij a_ic (ascending i), t = tau_j d,
// a_jc -= t v_0, a_ic -= t a_ij.  info = first column whose R diagonal is
// exactly zero (1-based), its reflector the identity.  The reference's own
// team-form QR is absent (aether-dsc); this order is the b200 build's, pinned
// by the oracle's restatement and against numpy's least squares.
template <int N, class T>
HK_FI void qr(const Team& tm, const TeamQr<T, N>& f, T* a, int m) {
    int info = 0;
    for (int j = 0; j < N; ++j) {
        T norm2 = T(0);
        for (int i = j; i < m; ++i) norm2 = norm2 + (a[i * N + j] * a[i * N + j]);
        const T ajj = a[j * N + j];
        tm.sync();                  // every thread has read the column before it changes
        if (!(norm2 > T(0))) {
            if (info == 0) info = j + 1;
            if (tm.rank == 0) {
                f.tau[j] = T(0);
                f.work[j] = T(0);
            }
            tm.sync();
            continue;
        }
        const T norm = math::sqrt(norm2);
        const T alpha = (ajj >= T(0)) ? -norm : norm;
        const T v0 = ajj - alpha;
        T vtv = v0 * v0;
        for (int i = j + 1; i < m; ++i) vtv = vtv + (a[i * N + j] * a[i * N + j]);
        const T tj = T(2) / vtv;
        for (int c = j + 1 + tm.rank; c < N; c += tm.size) {
            T d = v0 * a[j * N + c];
            for (int i = j + 1; i < m; ++i) d = d + (a[i * N + j] * a[i * N + c]);
            const T t = tj * d;
            a[j * N + c] = a[j * N + c] - (t * v0);
            for (int i = j + 1; i < m; ++i) a[i * N + c] = a[i * N + c] - (t * a[i * N + j]);
        }
        tm.sync();
        if (tm.rank == 0) {
            a[j * N + j] = alpha;
            f.tau[j] = tj;
            f.work[j] = v0;
        }
        tm.sync();
    }
    if (tm.rank == 0) *f.info = info;
    tm.sync();
}

// x = argmin |J x - r| from the factor (k right-hand sides, r m x k, x n x k,
// row-major): Q^T r by the reflectors in order, worked in place on r (the
// stage's own copy of it), then R x = (Q^T r)[0:n] backward, each row's dot
// product in ascending j; one thread per right-hand side; zeros for a
// rank-deficient factor.
template <int N, class T>
HK_FI void qrSolve(const Team& tm, const TeamQr<T, N>& f, int m, T* r, T* x, int k) {
    if (*f.info != 0) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = T(0);
        tm.sync();
        return;
    }
    const T* a = f.a;
    for (int c = tm.rank; c < k; c += tm.size) {
        for (int j = 0; j < N; ++j) {
            const T tj = f.tau[j], v0 = f.work[j];
            T d = v0 * r[j * k + c];
            for (int i = j + 1; i < m; ++i) d = d + (a[i * N + j] * r[i * k + c]);
            const T t = tj * d;
            r[j * k + c] = r[j * k + c] - (t * v0);
            for (int i = j + 1; i < m; ++i) r[i * k + c] = r[i * k + c] - (t * a[i * N + j]);
        }
        for (int q = 0; q < N; ++q) {
            const int i = N - 1 - q;
            T acc = r[i * k + c];
            for (int jj = i + 1; jj < N; ++jj) acc = acc - (a[i * N + jj] * x[jj * k + c]);
            x[i * k + c] = acc / a[i * N + i];
        }
    }
    tm.sync();
}

// x = (J^T J)^{-1} b from R (n x n upper triangle of the factor): R^T z = b
// forward, R x = z backward (ascending j in each dot product), in place when
// b == x; one thread per right-hand side; zeros for a rank-deficient factor.
template <int N, class T>
HK_FI void qrGramSolve(const Team& tm, const TeamQr<T, N>& f, const T* b, T* x, int k) {
    if (*f.info != 0) {
        for (int e = tm.rank; e < N * k; e += tm.size) x[e] = T(0);
        tm.sync();
        return;
    }
    const T* a = f.a;
    for (int c = tm.rank; c < k; c += tm.size) {
        for (int i = 0; i < N; ++i) {
            T acc = b[i * k + c];
            for (int jj = 0; jj < i; ++jj) acc = acc - (a[jj * N + i] * x[jj * k + c]);
            x[i * k + c] = acc / a[i * N + i];
        }
        for (int q = 0; q < N; ++q) {
            const int i = N - 1 - q;
            T acc = x[i * k + c];
            for (int jj = i + 1; jj < N; ++jj) acc = acc - (a[i * N + jj] * x[jj * k + c]);
            x[i * k + c] = acc / a[i * N + i];
        }
    }
    tm.sync();
}

// ------------------------------------------------------------ block sums

// The block of one key (a BlockSum, hawk/ir/team.py:544-600): entry (a, b) is
// the sum over the key's rows r = first .. first + rows - 1, in lane order
// from 0, of u[row a] * v[row b], where a lane holds `per` rows (row h of
// lane l at l * per + h; u rows of stride su, v rows of stride sv, sv = 0 for
// the constant 1); stored at out[a * ors + b * ocs].  The team's threads take
// entries; each entry's sum is one chain in lane order -- the same bits
// whatever the team.  An index map (an active-set build) is not built.
template <int P, int Q, class T>
HK_FI void blockSum(const Team& tm, T* out, const T* u, const T* v, std::size_t first, std::size_t rows,
                    std::size_t su, std::size_t sv, const void* index, std::size_t ors, std::size_t ocs, int per) {
    (void)index;
    for (int e = tm.rank; e < P * Q; e += tm.size) {
        const int a = e / Q, b = e % Q;
        T s = T(0);
        for (std::size_t r = 0; r < rows; ++r)
            for (int h = 0; h < per; ++h) {
                const std::size_t row = (first + r) * static_cast<std::size_t>(per) + static_cast<std::size_t>(h);
                s = s + (u[row * su + a] * v[row * sv + b]);
            }
        out[a * ors + b * ocs] = s;
    }
    tm.sync();
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

// ------------------------------------------------------ ordered sum, part 1

#if defined(__CUDA_ARCH__)
// One group of a plain ordered sum's first stage (hawk/emit/team.py:208-240):
// virtual lane t of group g adds the key's rows g * 1024 + t, + 65536, ... in
// order from +0, and the group's 1024 values fold by the halving tree
// s[i] += s[i + w] into sh[0].  A virtual lane past the key's rows holds +0,
// and a sum started at +0 is never -0 under round to nearest, so adding it is
// exact: the tree over the first `span` slots (the power of two covering the
// group's lanes that hold rows) makes the same bits as the tree over all
// 1024, and a group with no rows is +0 -- a key of 40 rows folds 64 slots in
// one group, not 64 groups of 1024.
template <class T>
HK_FI void orderedPart(const Team& tm, const T* u, std::size_t rows, std::size_t grp, T* sh) {
    const std::size_t first = grp * 1024;
    const std::size_t live = rows > first ? (rows - first < 1024 ? rows - first : 1024) : 0;
    if (live == 0) {
        if (tm.rank == 0) sh[0] = T(0);
        tm.sync();
        return;
    }
    std::size_t span = 1;
    while (span < live) span <<= 1;
    for (std::size_t t = static_cast<std::size_t>(tm.rank); t < span; t += static_cast<std::size_t>(tm.size)) {
        T acc = T(0);
        for (std::size_t r = first + t; r < rows; r += 65536) acc += u[r];
        sh[t] = acc;
    }
    tm.sync();
    for (std::size_t w = span >> 1; w > 0; w >>= 1) {
        for (std::size_t i = static_cast<std::size_t>(tm.rank); i < w; i += static_cast<std::size_t>(tm.size))
            sh[i] += sh[i + w];
        tm.sync();
    }
}
#endif

// ------------------------------------------------------- ordered scatter walk

#if defined(__CUDA_ARCH__)
// The walk of one lane chunk of an ordered scatter (hawk/emit/team.py:340-436)
// on one warp, for the keys it owns (key % G == g): log slots [lo, hi) in
// order, 32 a batch, eight batches loaded ahead.  The lanes of a batch holding
// the same owned key meet in one __match_any_sync group; the group's lowest
// lane adds the group's values into the key's bin in slot order.  So every
// bin gets its slots' values in slot order from its start -- the serial
// walk's operations, the same bits.  The bin of key c is
// bin[(c / div) * stride].  A key outside [0, cells) other than the skip key
// -1 adds nothing and sets `*flag`.
template <class T>
HK_FI void scatterWalk(const Team& tm, std::size_t lo, std::size_t hi, const std::int32_t* k, const T* v, T* bin,
                       std::size_t div, std::size_t stride, int G, int g, std::int32_t* flag, std::int64_t cells) {
    constexpr int kAhead = 8;
    const unsigned full = 0xffffffffu;
    const unsigned ln = static_cast<unsigned>(tm.rank) & 31u;
    unsigned bad = 0u;
    for (std::size_t b0 = lo; b0 < hi; b0 += 32 * kAhead) {
        std::int32_t key[kAhead];
        T val[kAhead];
#pragma unroll
        for (int a = 0; a < kAhead; ++a) {
            const std::size_t r = b0 + static_cast<std::size_t>(a) * 32 + ln;
            const bool in = r < hi;
            key[a] = in ? k[r] : -1;
            val[a] = in ? v[r] : T(0);
        }
#pragma unroll
        for (int a = 0; a < kAhead; ++a) {
            const bool inside = key[a] >= 0 && key[a] < cells;
            bad |= (!inside && key[a] != -1) ? 1u : 0u;
            const bool mine = inside && (key[a] % G) == g;
            const unsigned grp = __match_any_sync(full, mine ? key[a] : -1);
            const bool lead = mine && ln == static_cast<unsigned>(__ffs(grp) - 1);
            const std::size_t at = lead ? (static_cast<std::size_t>(key[a]) / div) * stride : 0;
            unsigned rest = lead ? grp : 0u;
            T acc = lead ? bin[at] : T(0);
            while (__any_sync(full, rest != 0u)) {
                const int src = rest != 0u ? __ffs(rest) - 1 : static_cast<int>(ln);
                const T x = __shfl_sync(full, val[a], src);
                if (rest != 0u) {
                    acc = acc + x;
                    rest &= rest - 1u;
                }
            }
            if (lead) bin[at] = acc;
            __syncwarp();           // the next batch's leader of a key reads this bin
        }
    }
    if (__any_sync(full, bad != 0u) && ln == 0u) *flag = 1;
    __syncwarp();
}

// An ordered scatter's chunk stage (hawk/ir/team.py:716-736) with G warps a
// chunk: team `lane` is warp g = lane % G of chunk lane / G (of count / G
// chunks over nSamples lanes, `slots` log slots a lane).  Warp g owns the
// keys c with c % G == g: up to 1024 cells in its shared bins (bin c / G),
// added onto the chunk's partial sum of each owned key afterwards; above
// that, in the chunk's column of the partial sums (zeroed by the first
// stage) directly.  Each partial sum is its chunk's values of the key in
// slot order from +0, as the reference's one warp a chunk makes it; the G
// warps only split the keys.  The slots are not put back to -1: the runtime
// refills the key log with -1 before every run (the plane's fill).  One team
// (warp) per block: the bins are the block's.
template <class T, int G>
HK_FI void scatterChunk(const Team& tm, long long lane, long long count, long long n_samples, int slots,
                        const std::int32_t* k, const T* v, T* p, std::int32_t* m) {
    __shared__ T bin[(1024 + G - 1) / G];
    const std::size_t chunks = static_cast<std::size_t>(count) / G;
    const std::size_t chunk = static_cast<std::size_t>(lane) / G;
    const int g = static_cast<int>(static_cast<std::size_t>(lane) % G);
    const std::size_t n = static_cast<std::size_t>(n_samples);
    const std::size_t span = (n + chunks - 1) / chunks;
    const std::size_t lo = chunk * span;
    const std::size_t hi = lo + span < n ? lo + span : n;
    const std::int64_t cells = m[0];
    std::int32_t* const flag = m + 1 + chunk;
    const std::size_t s = static_cast<std::size_t>(slots);
    if (cells <= 1024) {
        for (int j = tm.rank; j < (1024 + G - 1) / G; j += tm.size) bin[j] = T(0);
        tm.sync();
        scatterWalk<T>(tm, lo * s, hi * s, k, v, bin, G, 1, G, g, flag, cells);
        tm.sync();
        for (std::int64_t c = g + static_cast<std::int64_t>(G) * tm.rank; c < cells;
             c += static_cast<std::int64_t>(G) * tm.size)
            p[static_cast<std::size_t>(c) * chunks + chunk] += bin[static_cast<std::size_t>(c) / G];
    } else {
        scatterWalk<T>(tm, lo * s, hi * s, k, v, p + chunk, 1, chunks, G, g, flag, cells);
    }
    tm.sync();
}

// A reader stage's copy of a lane-major scratch plane (lane l's `comps`
// components contiguous at src[l * comps]) into a component-major output
// plane (component k of sample l at dst[k * pitch + l]), for the lanes
// [base, base + count): tile `tile` of the (lane tiles x component tiles)
// grid, 32 x 32 elements staged through `smem` (32 x 33 elements of T), so
// both the reads (one lane's 32 components) and the writes (one component of
// 32 lanes) are 32 consecutive elements a warp instruction.  Every thread of
// the block calls it for the same tile.
template <class T>
__device__ __forceinline__ void copyOutTile(const T* src, T* dst, unsigned long long pitch, long long comps,
                                            long long base, long long count, long long tile, unsigned char* smem) {
    T (*t)[33] = reinterpret_cast<T (*)[33]>(smem);
    const long long ktiles = (comps + 31) / 32;
    const long long lt = tile / ktiles, kt = tile - lt * ktiles;
    const int tx = static_cast<int>(threadIdx.x & 31u), rows = static_cast<int>(blockDim.x >> 5);
    for (int r = static_cast<int>(threadIdx.x >> 5); r < 32; r += rows) {
        const long long lane = lt * 32 + r, k = kt * 32 + tx;
        if (lane < count && k < comps) t[r][tx] = src[static_cast<std::size_t>(base + lane) * comps + k];
    }
    __syncthreads();
    for (int r = static_cast<int>(threadIdx.x >> 5); r < 32; r += rows) {
        const long long k = kt * 32 + r, lane = lt * 32 + tx;
        if (lane < count && k < comps) dst[static_cast<std::size_t>(k) * pitch + base + lane] = t[tx][r];
    }
    __syncthreads();
}
#endif

}  // namespace team

// ---------------------------------------------- the warp-form eigenvalues

namespace warp {

// The warp entry of an eigenvalues-only eigh (hawk/ir/team.py:236, the step
// `eigh_warp` of hawk/emit/team.py:492-505): one warp a lane, the values and
// the status of the one-thread form (hk/linalg.cuh eighValues: cyclic Jacobi,
// ascending values, info bits 1 and 2) with each rotation's row and column
// updates spread over the warp -- every element gets the one-thread form's
// operations in its order, so the same bits.  The working matrix lives in the
// block's shared scratch (one warp a block).
template <class T> struct EighValuesScratch {
    T s[32 * 32];
    T w[32];
    int info;
};

template <class T> struct EighValuesLane {
    T w;            // this lane's eigenvalue (ascending by lane)
    int info;
};

#if defined(__CUDA_ARCH__)
template <int N, class T>
HK_FI EighValuesLane<T> eighValues(EighValuesScratch<T>& sc, const T* a) {
    static_assert(N >= 1 && N <= 32, "the warp form holds up to 32 x 32");
    const T zero = T(0), one = T(1), half = T(0.5);
    const T eps = linalg::EighEps<T>::value();
    const int ln = static_cast<int>(threadIdx.x & 31u);
    T* const s = sc.s;
    for (int e = ln; e < N * N; e += 32) {
        const int i = e / N, j = e % N;
        s[e] = (j >= i) ? (half * a[i * N + j]) + (half * a[j * N + i]) : zero;
    }
    __syncwarp();
    if (N == 1) {
        if (ln == 0) {
            sc.w[0] = a[0];
            sc.info = 0;
        }
        __syncwarp();
        return {ln < N ? sc.w[ln] : zero, sc.info};
    }
    // the lower half mirrors the upper and the Frobenius sum, in the fill's order: one lane
    T fro2 = zero;
    if (ln == 0) {
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < N; ++j) {
                if (j < i) s[i * N + j] = s[j * N + i];
                fro2 = fro2 + (s[i * N + j] * s[i * N + j]);
            }
    }
    __syncwarp();
    for (int sweep = 0; sweep < linalg::eigh_sweeps(N); ++sweep)
        for (int p = 0; p < N - 1; ++p)
            for (int q = p + 1; q < N; ++q) {
                const T app = s[p * N + p], aqq = s[q * N + q], apq = s[p * N + q];
                __syncwarp();           // every lane has read the pivot block before it changes
                if (!(math::abs(apq) <= (eps * math::sqrt(math::abs(app * aqq))))) {
                    const T theta = (aqq - app) / (T(2) * apq);
                    const T sg = (theta < zero) ? T(-1) : one;
                    const T tn = sg / (math::abs(theta) + math::sqrt((theta * theta) + one));
                    const T cs = one / math::sqrt((tn * tn) + one);
                    const T sn = tn * cs;
                    if (ln == 0) {
                        s[p * N + p] = app - (tn * apq);
                        s[q * N + q] = aqq + (tn * apq);
                        s[p * N + q] = zero;
                        s[q * N + p] = zero;
                    }
                    for (int k = ln; k < N; k += 32) {
                        if ((k != p) && (k != q)) {
                            const T akp = s[k * N + p], akq = s[k * N + q];
                            const T np = (cs * akp) - (sn * akq);
                            const T nq = (sn * akp) + (cs * akq);
                            s[k * N + p] = np;
                            s[p * N + k] = np;
                            s[k * N + q] = nq;
                            s[q * N + k] = nq;
                        }
                    }
                }
                __syncwarp();
            }
    if (ln == 0) {
        int info = 0;
        T off2 = zero;
        for (int i = 0; i < N; ++i) {
            sc.w[i] = s[i * N + i];
            for (int j = 0; j < N; ++j)
                if (j != i) off2 = off2 + (s[i * N + j] * s[i * N + j]);
        }
        const T tol = static_cast<T>(N) * eps;
        if (!(off2 <= ((tol * tol) * fro2))) info = 1;
        for (int i = 0; i < N - 1; ++i) {
            int lo = i;
            for (int j = i + 1; j < N; ++j)
                if (sc.w[j] < sc.w[lo]) lo = j;
            if (lo != i) {
                const T tw = sc.w[i];
                sc.w[i] = sc.w[lo];
                sc.w[lo] = tw;
            }
        }
        const T gap = tol * math::sqrt(fro2);
        bool tight = false;
        for (int i = 0; i < N - 1; ++i)
            if (!((sc.w[i + 1] - sc.w[i]) > gap)) tight = true;
        sc.info = tight ? info + 2 : info;
    }
    __syncwarp();
    return {ln < N ? sc.w[ln] : zero, sc.info};
}
#endif

}  // namespace warp
}  // namespace linalg
}  // namespace hk
