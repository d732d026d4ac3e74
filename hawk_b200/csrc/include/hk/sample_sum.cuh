// hawk_b200 device library: reductions over samples.
//
// A kernel with SampleSum sinks (Param gradients of a VJP, hawk.sum/max/min
// cells) writes one row per 32 consecutive samples and column: the row is a
// fixed binary tree over the 32 lanes of a warp -- lanes paired across bit 4,
// then bit 3, ..., bit 0 -- whose nodes combine (sum, compensation) pairs
// (hawk/emit/wrapper.py:561-592, the host twin sampleSumRow_ and the device
// butterfly sampleSumWarp_ pair the same lanes).  A sum's node is
//     t = s + s2;  c = finite(t) ? (c + c2) + err(s, s2, t) : 0;  s = t
// with err the exact two-sum residual, larger magnitude first, +0 for a zero
// residual (hawk/_cells.py:44-49).  Max/min nodes keep the NaN-ignoring
// extreme of (lower lane, upper lane).
//
// Rows are then finished into the cell by the ``ordered`` tree of
// hawk/_cells.py:71-119: leaves of 4096 rows (256 slots x 16 terms, the terms
// of a slot added in order with a Neumaier step), a halving tree over the 256
// slots, then pairwise levels over the leaves (an odd last one carried up),
// and hi + comp at the root.  The device kernels that run that tree live in
// the runtime library; the node arithmetic is here so the two agree.
#pragma once
#include "base.cuh"

namespace hk {
namespace ss {

enum Op { kSum = 0, kMax = 1, kMin = 2 };

template <class T> HK_HD bool finite(T x) { return (x - x) == (x - x); }

// Exact residual a + b - s of s == fl(a + b), +0 for a zero residual.  The
// reference orders the operands by magnitude and takes Fast2Sum's
// small - (s - big); Knuth's 2Sum below needs no compare or select and yields
// the same exact residual for all finite a, b whose sum s does not overflow
// (Knuth, TAOCP vol. 2, 4.2.2 Theorem B; no intermediate of 2Sum overflows
// unless s does: Boldo, Graillat and Muller, ACM TOMS 44(1), 2017).  Where s
// is not finite the residual is discarded by every caller (the node's
// compensation becomes 0).  A zero residual is never -0: a round-to-nearest
// sum is -0 only when both operands are -0, here a - (s - bb) and b - bb,
// which needs a = b = -0 and s - bb = +0 -- but then s = -0, bb = +0 and
// s - bb = -0.  (The reference's Fast2Sum residual carries an explicit + 0.)
template <class T> HK_HD T two_sum_err(T a, T b, T s) {
    const T bb = s - a;
    return (a - (s - bb)) + (b - bb);
}

template <class T> HK_HD T extreme(int op, T a, T b) {
    if (a != a) return b;
    if (b != b) return a;
    return op == kMax ? (b > a ? b : a) : (b < a ? b : a);
}

template <class T> HK_HD T identity(int op) {
    if (op == kSum) return T(0);
    const T inf = T(1) / T(0);
    return op == kMax ? -inf : inf;
}

// A row node whose finiteness is checked once, at the row's root: a
// non-finite node makes every ancestor non-finite, so testing t at every node
// (as pair_combine does) and testing only the root's t give the same row --
// the root's compensation is zeroed by root_comp when its sum is not finite.
template <int OP, class T> HK_HD void pair_combine_unchecked(T& s, T& c, T s2, T c2) {
    if constexpr (OP != kSum) {
        s = extreme(OP, s, s2);
    } else {
        const T t = s + s2;
        c = (c + c2) + two_sum_err(s, s2, t);
        s = t;
    }
}
template <int OP, class T> HK_HD T root_comp(T s, T c) {
    return (OP != kSum || finite(s)) ? c : T(0);
}

// One node of a row: (s, c) of the lower lane joined with (s2, c2) of the upper.
template <int OP, class T> HK_HD void pair_combine(T& s, T& c, T s2, T c2) {
    if constexpr (OP != kSum) {
        s = extreme(OP, s, s2);
        return;
    } else {
        const T t = s + s2;
        const T e = two_sum_err(s, s2, t);
        c = finite(t) ? (c + c2) + e : T(0);
        s = t;
    }
}

// The finish tree's two node kinds (hawk/_cells.py:52-68).
template <int OP, class T> HK_HD void neumaier_add(T& h, T& c, T x, T xc) {
    if constexpr (OP == kSum) {
        const T s = h + x;
        const bool f = finite(s);
        c = f ? c + two_sum_err(h, x, s) : T(0);
        c = f ? c + xc : T(0);
        h = s;
    } else if constexpr (OP == kMax) {
        h = (h > x) ? h : x;
    } else {
        h = (h < x) ? h : x;
    }
}
template <int OP, class T> HK_HD void tree_join(T& h, T& c, T x, T xc) {
    if constexpr (OP == kSum) {
        const T s = h + x;
        c = finite(s) ? (c + xc) + two_sum_err(h, x, s) : T(0);
        h = s;
    } else if constexpr (OP == kMax) {
        h = (h > x) ? h : x;
    } else {
        h = (h < x) ? h : x;
    }
}

constexpr int kSlots = 256;
constexpr int kTerms = 16;
constexpr int kLeaf = kSlots * kTerms;   // rows per leaf

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
// One round of the halving butterfly: the lane holds M slots; the lower lane
// of the pair (bit `off` clear) keeps columns [0, M/2), the upper lane columns
// [M/2, M); each sends the other half to its partner and joins the kept column
// with the partner's copy into slot j.  A sum node is symmetric in its two
// operands (t = s + s2, the ordered two-sum residual, c + c2), so both lanes
// compute the same node without caring which holds the lower lane's value; a
// max/min node takes the lower lane's value first.  A lower lane's extra slot
// (M odd) is padding that only ever meets the same padding on later partners.
// FIRST (the round across bit 4): every compensation is still +0, so a sum
// node's (c + c2) + err is err exactly (err is never -0) and no compensation
// travels.
template <int M, int OP, bool FIRST = false, class T>
__device__ __forceinline__ void halve(T* h, T* c, int off, bool upper) {
    constexpr int LO = M / 2, UP = M - M / 2;
    const T pad = identity<T>(OP);
#pragma unroll
    for (int j = 0; j < UP; ++j) {
        const T lo_h = j < LO ? h[j] : pad;
        const T kh = upper ? h[LO + j] : lo_h;     // the column this lane keeps
        const T gh = upper ? lo_h : h[LO + j];     // the one it gives away
        const T rh = __shfl_xor_sync(0xffffffffu, gh, off);
        if constexpr (OP == kSum && FIRST) {
            const T t = kh + rh;
            c[j] = two_sum_err(kh, rh, t);
            h[j] = t;
            continue;
        }
        const T lo_c = j < LO ? c[j] : T(0);
        const T kc = upper ? c[LO + j] : lo_c;
        const T gc = upper ? lo_c : c[LO + j];
        const T rc = OP == kSum ? __shfl_xor_sync(0xffffffffu, gc, off) : T(0);
        T s = kh, sc = kc;
        if constexpr (OP == kSum) {
            pair_combine_unchecked<OP>(s, sc, rh, rc);
        } else {
            s = upper ? rh : kh;
            pair_combine_unchecked<OP>(s, sc, upper ? kh : rh, rc);
        }
        h[j] = s;
        c[j] = sc;
    }
}

// The rows of K consecutive 32-sample rows at once: every lane passes its
// samples' W terms for each of the K rows (h[q * W + k], identity past the
// last sample).  Each column's tree is the row tree above (lanes paired across
// bit 4, then 3, ..., 0), but each round a lane keeps only half of its columns,
// so a lane joins about K*W/16 pairs instead of 5*K*W.  Afterwards a lane
// holds at most ceil(K*W / 32) columns and calls store(col, sum, comp) for
// each, col = q * W + k.  All 32 lanes of the warp must call it.
template <int K, int W, int OP, class T, class Store>
__device__ __forceinline__ void rows_reduce(T (&h)[K * W], Store&& store) {
    constexpr int N = K * W;
    constexpr int M2 = N - N / 2, M3 = M2 - M2 / 2, M4 = M3 - M3 / 2, M5 = M4 - M4 / 2, M6 = M5 - M5 / 2;
    T c[N];
#pragma unroll
    for (int k = 0; k < N; ++k) c[k] = T(0);
    const unsigned lane = threadIdx.x & 31u;
    halve<N, OP, true>(h, c, 16, (lane & 16u) != 0u);
    halve<M2, OP>(h, c, 8, (lane & 8u) != 0u);
    halve<M3, OP>(h, c, 4, (lane & 4u) != 0u);
    halve<M4, OP>(h, c, 2, (lane & 2u) != 0u);
    halve<M5, OP>(h, c, 1, (lane & 1u) != 0u);
    // which columns this lane ended with: [first, first + held)
    int first = 0, held = N;
    auto keep = [&](bool upper, int half) {
        if (upper) {
            first += half;
            held -= half;
        } else if (held > half) {
            held = half;
        }
    };
    keep((lane & 16u) != 0u, N / 2);
    keep((lane & 8u) != 0u, M2 / 2);
    keep((lane & 4u) != 0u, M3 / 2);
    keep((lane & 2u) != 0u, M4 / 2);
    keep((lane & 1u) != 0u, M5 / 2);
#pragma unroll
    for (int j = 0; j < M6; ++j)
        if (j < held) store(first + j, h[j], root_comp<OP>(h[j], c[j]));
}

// The halving rounds across lane bits OFF, OFF / 2, ..., 1, starting from M
// columns a lane; FIRST as in halve (for the round that opens a row's tree).
template <int M, int OFF, int OP, bool FIRST, class T>
__device__ __forceinline__ void lane_rounds(T* h, T* c, unsigned lane) {
    if constexpr (OFF >= 1) {
        halve<M, OP, FIRST>(h, c, OFF, (lane & static_cast<unsigned>(OFF)) != 0u);
        lane_rounds<M - M / 2, OFF / 2, OP, false>(h, c, lane);
    }
}
template <int M, int OFF> constexpr int held_after() {
    if constexpr (OFF >= 1) return held_after<M - M / 2, OFF / 2>();
    else return M;
}

// The rows of K consecutive 32-sample rows with each row spread over P = 32 / K
// lanes: lane l holds, in slot q, sample (l % P) + P q of row l / P
// (h[q * W + k] for column k, identity past the last sample).  A row's tree
// pairs samples 16 apart first, then 8, ..., 1 (the row tree above); the
// levels whose pairs lie in one lane (16, ..., P apart: slots q and q + K/2,
// then q + K/4, ...) are joined in registers, the rest (P/2, ..., 1 apart) by
// the halving butterfly across lanes, starting from the W columns of the
// lane's row.  Every node joins the same two operands, lower sample first, as
// in rows_reduce, and after the in-register levels each lane holds exactly
// the columns rows_reduce's lane holds after as many rounds, so the rows are
// the same bits; the in-register levels take no shuffle and no select.
// store(col, sum, comp), col = row * W + k, as in rows_reduce.  All 32 lanes
// of the warp must call it.
template <int K, int W, int OP, class T, class Store>
__device__ __forceinline__ void rows_reduce_lanes(T (&h)[K * W], Store&& store) {
    constexpr int P = 32 / K;
    static_assert(K * P == 32, "K must be a power of two dividing 32");
    T c[K * W];
#pragma unroll
    for (int k = 0; k < K * W; ++k) c[k] = T(0);
    if constexpr (K >= 2) {
#pragma unroll
        for (int q = 0; q < K / 2; ++q)
#pragma unroll
            for (int k = 0; k < W; ++k) {
                T& s = h[q * W + k];
                const T s2 = h[(q + K / 2) * W + k];
                if constexpr (OP == kSum) {
                    const T t = s + s2;
                    c[q * W + k] = two_sum_err(s, s2, t);
                    s = t;
                } else {
                    s = extreme(OP, s, s2);
                }
            }
#pragma unroll
        for (int span = K / 4; span >= 1; span /= 2)
#pragma unroll
            for (int q = 0; q < span; ++q)
#pragma unroll
                for (int k = 0; k < W; ++k)
                    pair_combine_unchecked<OP>(h[q * W + k], c[q * W + k], h[(q + span) * W + k],
                                               c[(q + span) * W + k]);
    }
    const unsigned lane = threadIdx.x & 31u;
    lane_rounds<W, P / 2, OP, K == 1>(h, c, lane);
    int first = static_cast<int>(lane / P) * W, held = W, m = W;
#pragma unroll
    for (int off = P / 2; off >= 1; off /= 2) {
        if (lane & static_cast<unsigned>(off)) {
            first += m / 2;
            held -= m / 2;
        } else if (held > m / 2) {
            held = m / 2;
        }
        m -= m / 2;
    }
    constexpr int MF = held_after<W, P / 2>();
#pragma unroll
    for (int j = 0; j < MF; ++j)
        if (j < held) store(first + j, h[j], root_comp<OP>(h[j], c[j]));
}

#endif

}  // namespace ss
}  // namespace hk
