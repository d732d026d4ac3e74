// hawk_b200 device library: kernels that finish their own samples.
//
// A finishing kernel (a Terminated mask, hawk.finish) counts each sample that
// becomes finished in a launch into the one-cell uint32 `finished_count`
// lookup plane, and an automatic (steps="auto") kernel reads its trip budget
// from the one-cell `fused_steps` word (hawk/ir/nodes.py FINISHED_PLANE,
// FUSED_STEPS_PLANE; hawk/trace/steps.py).  The body calls
//   hawk_abi::finish_count(counter)  -- one newly finished sample;
//   hawk_clamp_count(word)           -- the word as a loop bound, <= INT_MAX.
#pragma once
#include "base.cuh"

// The budget word as an int trip count: values above INT_MAX run INT_MAX trips
// (the body clamps negative words to 0 before it asks).
HK_HD int hawk_clamp_count(long long n) { return n < 2147483647LL ? static_cast<int>(n) : 2147483647; }

namespace hawk_abi {

// One more finished sample in the counter cell.  The lanes of a warp that
// finish together add their count with ONE atomic (the count is only read
// after the launch, so the order of the increments does not matter).
template <class V> HK_FI void finish_count(const V& counter) {
    unsigned* cell = const_cast<unsigned*>(reinterpret_cast<const unsigned*>(counter.data()));
#if defined(__CUDA_ARCH__)
    const unsigned live = __activemask();
    const unsigned lane = threadIdx.x & 31u;
    if (lane == static_cast<unsigned>(__ffs(live) - 1)) atomicAdd(cell, static_cast<unsigned>(__popc(live)));
#else
    *cell += 1u;
#endif
}

}  // namespace hawk_abi

namespace hk {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
// The persistent entry's report, once per warp after its loop (all 32 lanes
// converged): the longest per-sample trip count into `steps` (max), the steps
// run into `stepsum` and util[0] (sums); each pointer may be null.
HK_FI void persist_report(unsigned* steps, unsigned long long* stepsum, unsigned long long* util,
                          unsigned longest, unsigned long long ran) {
    const unsigned top = __reduce_max_sync(0xffffffffu, longest);
    unsigned long long total = ran;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if ((threadIdx.x & 31u) == 0u) {
        if (steps != nullptr && top != 0u) atomicMax(steps, top);
        if (total != 0ull) {
            if (stepsum != nullptr) atomicAdd(stepsum, total);
            if (util != nullptr) atomicAdd(&util[0], total);
        }
    }
}

// The warp's finished samples (finishing in the launch or on entry) into the
// finished counter cell, one atomic per warp.
template <class V> HK_FI void persist_finished(const V& counter, unsigned fin) {
    const unsigned total = __reduce_add_sync(0xffffffffu, fin);
    if ((threadIdx.x & 31u) == 0u && total != 0u)
        atomicAdd(const_cast<unsigned*>(reinterpret_cast<const unsigned*>(counter.data())), total);
}
#endif

}  // namespace hk
