// hawk_b200 device library: the by-value argument mirrors of an emitted entry.
//
// Every emitted ``__global__`` entry takes its planes as these PODs, by value,
// in the kernel's ``arg_spec`` order, followed by the int64 partition triple
// ``(base, count, nSamples)``.  Sizes and field order are the reference's
// (hawk/_contracts.py:58-92; the bind rule is src/hawk_core.cpp:228-258), so a
// host runtime that packs a slot for the reference's entries packs it for
// these: a GRef plane's component pitch is ``samples * stride``.
#pragma once
#include "base.cuh"

namespace hk {
namespace abi {

// A Vector/Matrix plane: component-major SoA, unit sample stride.
struct GRefMirror {
    double* data_;
    u64 samples_;
    u64 compStride_;     // elements between component k and k+1 of one sample
    u64 sampleStride_;   // elements between samples (1 for every hawk plane)
    i32 deviceType_;     // DLPack device code (2 = CUDA)
    i32 deviceId_;
};

// A per-sample scalar plane, a one-cell lookup plane, or a row plane.
struct ScalarHandle {
    void* data;
    u64 samples;
    u64 stride;
    i32 deviceType;
    i32 deviceId;
};

// The integer twin of ScalarHandle (an int32 Mutable, an int lookup).
struct IntHandle {
    void* data;
    u64 samples;
    u64 stride;
    i32 deviceType;
    i32 deviceId;
};

struct PartitionTriple {
    i64 base;
    i64 count;
    i64 nSamples;
};

static_assert(sizeof(GRefMirror) == 40, "GRefMirror is 40 bytes");
static_assert(sizeof(ScalarHandle) == 32, "ScalarHandle is 32 bytes");
static_assert(sizeof(IntHandle) == 32, "IntHandle is 32 bytes");
static_assert(sizeof(PartitionTriple) == 24, "PartitionTriple is 24 bytes");

// The index type the nsamples role is passed as (EAGLE_ABI_INDEX_T, 8 bytes).
typedef u64 index_t;

}  // namespace abi
}  // namespace hk
