// hawk_b200 device library: shared-memory stages filled by the TMA unit.
//
// A CTA streams its tiles of input planes through S shared-memory stages:
// thread 0 issues one bulk copy per plane component and tile
// (cp.async.bulk global -> shared, completion counted in bytes on the stage's
// "full" mbarrier); every warp waits for the stage, computes from shared
// memory, and arrives on the stage's "empty" mbarrier; thread 0 waits for
// "empty" before refilling the stage with the tile S ahead.  The loads of the
// next S - 1 tiles are in flight while the CTA computes, whatever the compute
// costs, and the copies need no registers.
//
// Every wait is bounded in time (kWaitNs of the global timer).  A wait that
// runs out sets a bit in the unit's hk_error_flags word and the caller stops
// its loop; before the CTA exits, thread 0 waits (bounded again) for the
// copies it issued, so no copy is left writing shared memory.  The host reads
// and clears the word through hkb_library_errors.
#pragma once
#include "base.cuh"

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
extern "C" __device__ unsigned int hk_error_flags;
#endif

namespace hk {
namespace stage {

// Error bits of hk_error_flags.
constexpr unsigned kErrFullWait = 1u;    // a stage's data did not arrive in time
constexpr unsigned kErrEmptyWait = 2u;   // a stage was not released in time
constexpr unsigned kErrDrain = 4u;       // copies still in flight when the CTA gave up
constexpr unsigned kErrWarpWait = 16u;   // a warp's tile did not arrive in time; it read global memory

// Bound of one wait: two seconds.
constexpr unsigned long long kWaitNs = 2000000000ull;

#if defined(__CUDA_ARCH__)
HK_FI unsigned smem(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

HK_FI unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

HK_FI void init(unsigned long long* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem(bar)), "r"(count) : "memory");
}

// Makes the barrier initialisations visible to the TMA unit (async proxy).
HK_FI void fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

HK_FI void arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem(bar)), "r"(bytes)
                 : "memory");
}

HK_FI void arrive(unsigned long long* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem(bar)) : "memory");
}

HK_FI bool try_wait(unsigned long long* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}

// Wait for the phase with `parity` to complete; false when kWaitNs passed first.
HK_FI bool wait(unsigned long long* bar, unsigned parity) {
    if (try_wait(bar, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!try_wait(bar, parity))
        if (now_ns() - t0 > kWaitNs) return false;
    return true;
}

// `bytes` (a multiple of 16, both addresses 16-byte aligned) from global memory
// into shared memory, counted on `bar`.
HK_FI void copy(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem(dst)),
                 "l"(__cvta_generic_to_global(src)), "r"(bytes), "r"(smem(bar))
                 : "memory");
}

HK_FI void fail(unsigned bit) { atomicOr(&hk_error_flags, bit); }

// Orders this thread's earlier generic-proxy accesses to shared memory before
// later async-proxy (bulk copy) writes to it.
HK_FI void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
#endif

// Whether a plane component can be copied in tiles: 16-byte aligned start and
// a component pitch and partition base that keep every tile 16-byte aligned.
HK_HD bool aligned(const void* p, unsigned long long pitch_bytes, long long base_bytes) {
    return (reinterpret_cast<unsigned long long>(p) & 15ull) == 0ull && (pitch_bytes & 15ull) == 0ull &&
           (static_cast<unsigned long long>(base_bytes) & 15ull) == 0ull;
}

#if defined(__CUDA_ARCH__)
// The stages of one CTA: S full barriers, S empty barriers, then S buffers of
// `stage_bytes` (a multiple of 128) in the CTA's dynamic shared memory.
template <int S>
struct Pipe {
    unsigned long long* full;
    unsigned long long* empty;
    unsigned char* buf;
    unsigned stage_bytes;    // the stride of the stage buffers
    unsigned tx_bytes;       // the bytes one fill copies (what the full barrier expects)
    unsigned issued = 0u;    // thread 0: bit s set once stage s was filled
    unsigned parity = 0u;    // thread 0: bit s = parity of stage s's last fill

    HK_FI Pipe(unsigned char* shared, unsigned stride, unsigned bytes) {
        full = reinterpret_cast<unsigned long long*>(shared);
        empty = full + S;
        buf = shared + 128;
        stage_bytes = stride;
        tx_bytes = bytes;
    }

    // Thread 0 initialises the barriers; every thread of the CTA must call it.
    HK_FI void setup(unsigned consumers) {
        if (threadIdx.x == 0) {
#pragma unroll
            for (int s = 0; s < S; ++s) {
                init(full + s, 1u);
                init(empty + s, consumers);
            }
            fence_init();
        }
        __syncthreads();
    }

    HK_FI unsigned char* stage(int s) const { return buf + static_cast<unsigned long long>(s) * stage_bytes; }

    // Thread 0: fill stage s with a tile through `issue(stage pointer, barrier)`,
    // which makes the tile's bulk copies on the barrier; first waits for the
    // stage's previous use (the j-th tile, j >= S) to be released.
    template <class Issue>
    HK_FI bool fill(long long j, Issue&& issue) {
        const int s = static_cast<int>(j % S);
        if (j >= S && !wait(empty + s, static_cast<unsigned>(((j - S) / S) & 1))) {
            hk::stage::fail(kErrEmptyWait);
            return false;
        }
        arrive_expect_tx(full + s, tx_bytes);
        issue(stage(s), full + s);
        const unsigned bit = 1u << s;
        issued |= bit;
        parity = ((j / S) & 1) ? (parity | bit) : (parity & ~bit);
        return true;
    }

    // Every consumer: wait for the j-th tile's stage; nullptr when it timed out.
    // (The caller makes the outcome warp-uniform before any warp-wide step.)
    HK_FI const unsigned char* acquire(long long j) {
        const int s = static_cast<int>(j % S);
        if (!wait(full + s, static_cast<unsigned>((j / S) & 1))) {
            hk::stage::fail(kErrFullWait);
            return nullptr;
        }
        return stage(s);
    }

    // One lane of every consuming warp: the warp is done with the j-th tile's stage.
    HK_FI void release(long long j) {
        __syncwarp();
        if ((threadIdx.x & 31u) == 0u) arrive(empty + static_cast<int>(j % S));
    }

    // Thread 0, before the CTA exits after an error: wait (bounded) for the
    // copies it issued, so none is left writing shared memory.
    HK_FI void drain() {
#pragma unroll
        for (int s = 0; s < S; ++s)
            if (((issued >> s) & 1u) && !wait(full + s, (parity >> s) & 1u)) hk::stage::fail(kErrDrain);
    }
};

// One warp's own tile of inputs, fetched one trip ahead: the warp's lane 0
// issues the next trip's bulk copies on the warp's mbarrier before the warp
// reduces the current trip, so the copies overlap the reduction and need no
// registers; no other warp takes part, so nothing waits across warps.  The
// block's dynamic shared memory holds the warps' barriers in its first 128
// bytes, then one `stage_bytes` tile per warp.
//
// A tile that does not arrive within kWaitNs is not waited for again: the warp
// sets kErrWarpWait, reads that trip's inputs and every later trip's from
// global memory (the same values, so the outputs are complete), issues no more
// copies, and before it returns waits once more (bounded) for the copy still
// landing, setting kErrDrain if it never does.
struct WarpTile {
    unsigned long long* bar;
    unsigned char* buf;
    unsigned tx_bytes;
    unsigned parity = 0u;
    bool pending = false;    // a fill has been issued and not yet taken
    bool broken = false;     // a wait ran out: no more fills

    // Every lane of the warp calls it.
    HK_FI WarpTile(unsigned char* shared, unsigned stage_bytes, unsigned tx) {
        const unsigned w = threadIdx.x >> 5;
        bar = reinterpret_cast<unsigned long long*>(shared) + w;
        buf = shared + 128 + static_cast<unsigned long long>(w) * stage_bytes;
        tx_bytes = tx;
        if ((threadIdx.x & 31u) == 0u) {
            init(bar, 1u);
            fence_init();
        }
        __syncwarp();
    }

    // Every lane: fill the tile through `issue(tile, barrier)`, run by lane 0
    // (the tile's bulk copies on the barrier).  The warp's earlier reads of the
    // tile are ordered before the copies' writes.
    template <class Issue>
    HK_FI void fill(Issue&& issue) {
        if (broken) return;
        __syncwarp();
        fence_proxy_async();
        if ((threadIdx.x & 31u) == 0u) {
            arrive_expect_tx(bar, tx_bytes);
            issue(buf, bar);
        }
        pending = true;
    }

    // Every lane: the filled tile, or nullptr (none pending, or its wait ran
    // out) -- the caller then reads global memory.
    HK_FI const unsigned char* acquire() {
        if (!pending || broken) return nullptr;
        if (__all_sync(0xffffffffu, wait(bar, parity))) {
            parity ^= 1u;
            pending = false;
            return buf;
        }
        broken = true;
        if ((threadIdx.x & 31u) == 0u) fail(kErrWarpWait);
        return nullptr;
    }

    // Every lane, before the warp returns: a copy still landing is waited for.
    HK_FI void finish() {
        if (pending && (threadIdx.x & 31u) == 0u && !wait(bar, parity)) fail(kErrDrain);
        __syncwarp();
    }
};
#endif

}  // namespace stage
}  // namespace hk
