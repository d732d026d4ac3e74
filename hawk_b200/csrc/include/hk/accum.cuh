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
    auto* slot = target.data() + at.g;
    using E = typename hk::detail::Pointee<decltype(slot)>::type;
    atomicAdd(slot, static_cast<E>(term));
}

template <class V, class T>
HK_FI void accum_add_compensated(const V& target, const V& comp, const hk::SampleIndex& at, T term) {
    auto* slot = target.data() + at.g;
    using E = typename hk::detail::Pointee<decltype(slot)>::type;
    atomic_add_compensated(slot, comp.data() + at.g, static_cast<E>(term));
}

template <class V, class T> HK_FI void accum_or(const V& target, const hk::SampleIndex& at, T bits) {
    atomicOr(reinterpret_cast<unsigned*>(target.data() + at.g), static_cast<unsigned>(bits));
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

// Aligned groups of W lanes whose keys are equal: each group's total, one
// commit per group.  False (nothing committed) when the warp is not fully
// converged or a group's keys differ.
template <int W, class E> HK_FI bool groups(E* target, E* comp, long long key, E term) {
    static_assert(W >= 1 && W <= 32 && (W & (W - 1)) == 0, "a run is a power-of-two number of lanes");
    if (__activemask() != kFull) return false;
    const unsigned lane = threadIdx.x & 31u;
    const long long lead = __shfl_sync(kFull, key, static_cast<int>(lane & ~static_cast<unsigned>(W - 1)));
    if (!__all_sync(kFull, lead == key)) return false;
    E v = term;
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    if ((lane & static_cast<unsigned>(W - 1)) == 0u) commit(target + key, comp == nullptr ? comp : comp + key, v);
    return true;
}

// Keys non-decreasing along the warp: each run of equal keys sums to its first
// lane (a segmented doubling sum), which commits.  False when the warp is not
// fully converged or its keys are not sorted.
template <class E> HK_FI bool sorted_runs(E* target, E* comp, long long key, E term) {
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
    if (lane == 0u || prev != key) commit(target + key, comp == nullptr ? comp : comp + key, v);
    return true;
}

template <class V> HK_FI auto slot_of(const V& v) -> decltype(v.data()) { return v.data(); }

template <int W, class V, class T>
HK_FI void add(const V& target, const SampleIndex& at, T term, const SampleIndex&, State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!groups<W, E>(target.data(), static_cast<E*>(nullptr), at.g, static_cast<E>(term)))
        atomicAdd(target.data() + at.g, static_cast<E>(term));
}

template <int W, class V, class T>
HK_FI void addCompensated(const V& target, const V& comp, const SampleIndex& at, T term, const SampleIndex&,
                          State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!groups<W, E>(target.data(), comp.data(), at.g, static_cast<E>(term)))
        hawk_abi::atomic_add_compensated(target.data() + at.g, comp.data() + at.g, static_cast<E>(term));
}

template <class V, class T> HK_FI void addTested(const V& target, const SampleIndex& at, T term, State& s) {
    add<32>(target, at, term, at, s);
}

template <class V, class T>
HK_FI void addTestedCompensated(const V& target, const V& comp, const SampleIndex& at, T term, State& s) {
    addCompensated<32>(target, comp, at, term, at, s);
}

template <class V, class T> HK_FI void addSorted(const V& target, const SampleIndex& at, T term, State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!sorted_runs<E>(target.data(), static_cast<E*>(nullptr), at.g, static_cast<E>(term)))
        atomicAdd(target.data() + at.g, static_cast<E>(term));
}

template <class V, class T>
HK_FI void addSortedCompensated(const V& target, const V& comp, const SampleIndex& at, T term, State&) {
    using E = typename detail::Pointee<decltype(slot_of(target))>::type;
    if (!sorted_runs<E>(target.data(), comp.data(), at.g, static_cast<E>(term)))
        hawk_abi::atomic_add_compensated(target.data() + at.g, comp.data() + at.g, static_cast<E>(term));
}
#endif

}  // namespace run
}  // namespace accum
}  // namespace hk
