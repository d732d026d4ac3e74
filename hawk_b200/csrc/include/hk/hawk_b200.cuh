// hawk_b200 device library: everything an emitted b200 translation unit includes.
//
// An emitted unit is: this header, the scalar-mode aliases (Real, Int), the
// self-check exports, and one ``extern "C" __global__`` entry per kernel whose
// body is the reference renderer's per-sample text.  The entry's frame is one
// of the two below; the launch geometry (grid, block, stream) is the runtime's.
//
//  * the lane frame: a grid-stride loop over the partition's samples, one
//    sample per thread per trip, consecutive threads on consecutive samples;
//  * the row frame (kernels with sample sums): a grid-stride loop over rows of
//    32 consecutive samples, one warp per row per trip, lane l on sample
//    32*row + l, closed by the warp's row reduction (sample_sum.cuh).
#pragma once
#include "base.cuh"
#include "abi.cuh"
#include "math.cuh"
#include "item.cuh"
#include "views.cuh"
#include "linalg.cuh"
#include "ints.cuh"
#include "sample_sum.cuh"
#include "stage.cuh"
#include "steps.cuh"
#include "accum.cuh"
#include "team.cuh"

namespace hk {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
// The lane frame's first sample and stride.
HK_FI i64 lane_first() { return static_cast<i64>(blockIdx.x) * blockDim.x + threadIdx.x; }
HK_FI i64 lane_step() { return static_cast<i64>(gridDim.x) * blockDim.x; }
// The row frame's first row and stride (one warp per row).
HK_FI i64 warp_first() { return lane_first() >> 5; }
HK_FI i64 warp_step() { return lane_step() >> 5; }
#endif

}  // namespace hk

// The dynamic shared memory every block of the unit's entry uses, exported
// for the loader, which sets the entry's limit and passes it at launch (a
// unit that exports nothing uses none).
#define HK_DYNAMIC_SMEM(BYTES) extern "C" __device__ const unsigned int hk_dynamic_smem_bytes = (BYTES);

// The layout self-check exports: the loader reads them and refuses a unit whose
// mirrors are not the sizes it packs (hawk/artifact/layout.py:35-61).  Every
// unit also defines its error word, which a bounded wait that ran out sets
// (hk/stage.cuh) and the host reads with hkb_library_errors.
#define HK_ABI_TAG "aether-abi/2"
#define HK_SELF_CHECK_EXPORTS                                                        \
    extern "C" __device__ unsigned int hk_error_flags = 0u;                          \
    extern "C" __device__ const char eagle_abi_tag[] = HK_ABI_TAG;                   \
    extern "C" __device__ unsigned long long eagle_layout_sizes[5] = {               \
        sizeof(hk::abi::GRefMirror), sizeof(hk::abi::ScalarHandle),                  \
        sizeof(hk::abi::IntHandle), sizeof(hk::abi::index_t),                        \
        sizeof(hk::abi::PartitionTriple)};
