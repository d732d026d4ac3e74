// hawk_b200 device library: scattered commits (hawk.scatter, the VJP of a gather).
//
// A scattered commit adds a sample's term into a slot of a plane chosen by a
// key: `hawk.scatter(acc, policy=...)[key] += x`, or the adjoint of a table
// read `table[idx]`, which adds into bar_table[idx] (hawk/trace/reduce.py,
// hawk/trace/value.py by_key).  Many samples meet on one slot, so every commit
// is an atomic read-modify-write, as on the reference's device and host-team
// targets (hawk/emit/wrapper.py:392-437, :1068-1085): the order of the adds is
// the hardware's, and the sum contract is the reference's -- within a bound of
// eps * sum|t| of the exact sum per slot (tests/test_keyed_commit.py).
//
//   hawk_abi::accum_add(t, at, x)                 t[at] += x
//   hawk_abi::accum_add_compensated(t, c, at, x)  t[at] += x; c[at] += the add's
//                                                 rounding error (2Sum of the
//                                                 old value and x)
//   hawk_abi::accum_or(t, at, bits)               t[at] |= bits (32-bit words)
//   hawk_abi::fold_companion(t, c, at)            t += c, c = the residual
//
// A key the tracer proves constant over aligned runs of lanes, tests per warp
// or reads from a Sorted index commits through hk::accum::run (the reference
// spells aether::accum::run there): the lanes of a run add their terms in the
// warp (shuffles, no shared memory) and ONE lane commits the run's total.  The
// run is verified here before it is used -- equal keys over each aligned group
// of W lanes (add<W>), over the whole warp (addTested), or non-decreasing keys
// along the warp (addSorted: one commit per run of equal keys) -- on a fully
// converged warp; otherwise every lane commits its own term, which is always
// correct.  A run's total is a tree sum, so its bits may differ from a serial
// sum's; the contract above covers both.
#pragma once
#include "base.cuh"
#include "views.cuh"
#include "sample_sum.cuh"

namespace hk {
namespace detail {
template <class P> struct Pointee;
template <class T> struct Pointee<T*> { typedef T type; };
}  // namespace detail
}  // namespace hk

namespace hk {
namespace accum {

// A scatter target a block commits into through a private copy in its shared
// memory (when the plane fits the entry's share): commits land in the copy at
// shared-memory atomic rates, and the block adds its copy into the plane once,
// slot by slot, when it leaves (flush_*).  A key past the copy commits to the
// plane directly.  `n` is the plane's slots.
template <class T> struct PrivOut {
    T* global;
    T* local;
    u64 n;
    bool priv;
    HK_HD T* data() const { return global; }
    HK_HD u64 samples() const { return n; }
};

// The slot of key k: the plane's, or a private copy's.
template <class V> HK_HD auto slot(const V& v, i64 k) -> decltype(v.data()) { return v.data() + k; }
template <class T> HK_HD T* slot(const PrivOut<T>& v, i64 k) {
    return (v.priv && static_cast<u64>(k) < v.n) ? v.local + k : v.global + k;
}

}  // namespace accum
}  // namespace hk

namespace hawk_abi {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
template <class E> HK_FI void atomic_add_compensated(E* slot, E* comp, E t) {
    const E old = atomicAdd(slot, t);
    const E s = old + t;                        // the value the atomic stored (one rounding)
    if (hk::ss::finite(s)) {
        const E e = hk::ss::two_sum_err(old, t, s);
        if (e != E(0)) atomicAdd(comp, e);
    }
}

template <class V, class T> HK_FI void accum_add(const V& target, const hk::SampleIndex& at, T term) {
    auto* slot = hk::accum::slot(target, at.g);
    using E = typename hk::detail::Pointee<decltype(slot)>::type;
    atomicAdd(slot, static_cast<E>(term));
}

template <class V, class C, class T>
HK_FI void accum_add_compensated(const V& target, const C& comp, const hk::SampleIndex& at, T term) {
    auto* slot = hk::accum::slot(target, at.g);
    using E = typename hk::detail::Pointee<decltype(slot)>::type;
    atomic_add_compensated(slot, hk::accum::slot(comp, at.g), static_cast<E>(term));
}

template <class V, class T> HK_FI void accum_or(const V& target, const hk::SampleIndex& at, T bits) {
    atomicOr(reinterpret_cast<unsigned*>(hk::accum::slot(target, at.g)), static_cast<unsigned>(bits));
}
#endif

// One slot of a target and its companion: the target takes the compensated
// sum, the companion the residual (none for a non-finite sum).
template <class V> HK_HD void fold_companion(const V& target, const V& comp, const hk::SampleIndex& at) {
    auto& t = target.data()[at.g];
    auto& c = comp.data()[at.g];
    const auto s = t + c;
    const auto e = hk::ss::two_sum_err(t, c, s);
    t = s;
    c = hk::ss::finite(s) ? e : decltype(s)(0);
}

}  // namespace hawk_abi

namespace hk {
namespace accum {
namespace run {

// The run state the entry declares per target: the device commits per warp, so
// nothing is carried from one sample to the next.
struct State {};

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
constexpr unsigned kFull = 0xffffffffu;

template <class E> HK_FI void commit(E* slot, E* comp, E v) {
    if (comp != nullptr) hawk_abi::atomic_add_compensated(slot, comp, v);
    else atomicAdd(slot, v);
}

// The slot of key k in a target or its companion (none: null).
template <class V> HK_FI auto at_key(const V& v, i64 k) -> decltype(slot(v, k)) { return slot(v, k); }
struct NoComp {};
template <class E> HK_FI E* at_key_comp(const NoComp&, i64) { return nullptr; }
template <class E, class V> HK_FI E* at_key_comp(const V& v, i64 k) { return slot(v, k); }

// Aligned groups of W lanes whose keys are equal: each group's total, one
// commit per group.  False (nothing committed) when the warp is not fully
// converged or a group's keys differ.
template <int W, class E, class V, class C> HK_FI bool groups(const V& target, const C& comp, long long key, E term) {
    static_assert(W >= 1 && W <= 32 && (W & (W - 1)) == 0, "a run is a power-of-two number of lanes");
    if (__activemask() != kFull) return false;
    const unsigned lane = threadIdx.x & 31u;
    const long long lead = __shfl_sync(kFull, key, static_cast<int>(lane & ~static_cast<unsigned>(W - 1)));
    if (!__all_sync(kFull, lead == key)) return false;
    E v = term;
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    if ((lane & static_cast<unsigned>(W - 1)) == 0u) commit(at_key(target, key), at_key_comp<E>(comp, key), v);
    return true;
}

// Keys non-decreasing along the warp: each run of equal keys sums to its first
// lane (a segmented doubling sum), which commits.  False when the warp is not
// fully converged or its keys are not sorted.
template <class E, class V, class C> HK_FI bool sorted_runs(const V& target, const C& comp, long long key, E term) {
    if (__activemask() != kFull) return false;
    const unsigned lane = threadIdx.x & 31u;
    const long long prev = __shfl_up_sync(kFull, key, 1);
    if (!__all_sync(kFull, lane == 0u || prev <= key)) return false;
    E v = term;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const E u = __shfl_down_sync(kFull, v, o);
        const long long k2 = __shfl_down_sync(kFull, key, o);
        if (lane + static_cast<unsigned>(o) < 32u && k2 == key) v += u;
    }
    if (lane == 0u || prev != key) commit(at_key(target, key), at_key_comp<E>(comp, key), v);
    return true;
}

template <class V> HK_FI auto slot_of(const V& v) -> decltype(v.data()) { return v.data(); }

template <int W, class V, class T>
HK_FI void add(const V& target, const SampleIndex& at, T term, const SampleIndex&, State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!groups<W, E>(target, NoComp{}, at.g, static_cast<E>(term))) atomicAdd(slot(target, at.g), static_cast<E>(term));
}

template <int W, class V, class C, class T>
HK_FI void addCompensated(const V& target, const C& comp, const SampleIndex& at, T term, const SampleIndex&,
                          State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!groups<W, E>(target, comp, at.g, static_cast<E>(term)))
        hawk_abi::atomic_add_compensated(slot(target, at.g), slot(comp, at.g), static_cast<E>(term));
}

template <class V, class T> HK_FI void addTested(const V& target, const SampleIndex& at, T term, State& s) {
    add<32>(target, at, term, at, s);
}

template <class V, class C, class T>
HK_FI void addTestedCompensated(const V& target, const C& comp, const SampleIndex& at, T term, State& s) {
    addCompensated<32>(target, comp, at, term, at, s);
}

template <class V, class T> HK_FI void addSorted(const V& target, const SampleIndex& at, T term, State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!sorted_runs<E>(target, NoComp{}, at.g, static_cast<E>(term))) atomicAdd(slot(target, at.g), static_cast<E>(term));
}

template <class V, class C, class T>
HK_FI void addSortedCompensated(const V& target, const C& comp, const SampleIndex& at, T term, State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!sorted_runs<E>(target, comp, at.g, static_cast<E>(term)))
        hawk_abi::atomic_add_compensated(slot(target, at.g), slot(comp, at.g), static_cast<E>(term));
}

#endif

}  // namespace run

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
// ------------------------------------------------- block-private scatter targets

// The shared-memory share of an entry whose targets a block privatises: the
// block's dynamic shared memory, handed out target by target in unpack order.
struct PrivSpace {
    unsigned char* base;
    unsigned bytes;
    unsigned used;
};

HK_FI PrivSpace private_space() {
    extern __shared__ __align__(16) unsigned char hk_priv_dyn[];
    unsigned r;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
    return PrivSpace{hk_priv_dyn, r, 0u};
}

// A block's private copy of the target `v` (zeroed), when the rest of its
// share holds the plane's slots; else the plane itself.  Every thread of the
// block makes the same calls in the same order, then the block waits
// (__syncthreads) before its first commit.
template <class T> HK_FI PrivOut<T> privatise(PrivSpace& sp, const ScalarOut<T>& v) {
    PrivOut<T> o{v.p, nullptr, v.n, false};
    const unsigned long long need = (v.n * sizeof(T) + 15ull) & ~15ull;
    if (v.n > 0 && sp.used + need <= sp.bytes) {
        o.local = reinterpret_cast<T*>(sp.base + sp.used);
        o.priv = true;
        sp.used += static_cast<unsigned>(need);
        for (u64 k = threadIdx.x; k < v.n; k += blockDim.x) o.local[k] = T(0);
    }
    return o;
}

// The block's copies into the planes, after every commit of the block
// (__syncthreads first): a plain target adds each nonzero slot, a compensated
// one commits each slot with the compensated add and adds its companion's
// slot, an OR target ORs each nonzero word.
template <class T> HK_FI void flush_add(const PrivOut<T>& o) {
    if (!o.priv) return;
    for (u64 k = threadIdx.x; k < o.n; k += blockDim.x) {
        const T v = o.local[k];
        if (v != T(0)) atomicAdd(o.global + k, v);
    }
}

template <class T> HK_FI void flush_compensated(const PrivOut<T>& o, const PrivOut<T>& c) {
    for (u64 k = threadIdx.x; k < o.n; k += blockDim.x) {
        if (o.priv) {
            const T v = o.local[k];
            if (v != T(0)) hawk_abi::atomic_add_compensated(o.global + k, c.global + k, v);
        }
        if (c.priv && k < c.n) {
            const T e = c.local[k];
            if (e != T(0)) atomicAdd(c.global + k, e);
        }
    }
}

template <class T> HK_FI void flush_or(const PrivOut<T>& o) {
    if (!o.priv) return;
    for (u64 k = threadIdx.x; k < o.n; k += blockDim.x) {
        const unsigned v = static_cast<unsigned>(o.local[k]);
        if (v != 0u) atomicOr(reinterpret_cast<unsigned*>(o.global + k), v);
    }
}
#endif
}  // namespace accum
}  // namespace hk
