// hawk_b200 device library: base definitions.
//
// The library is compiled by NVRTC (sm_100a) inside each emitted translation
// unit, and NVRTC carries no C/C++ standard headers.  Everything below is
// therefore self-contained: the few fixed-width integer names the emitted body
// text spells (``std::int32_t`` and friends) are declared here when the unit is
// compiled by NVRTC, and taken from <cstdint> under nvcc or a host compiler.
#pragma once

#if defined(__CUDACC_RTC__)
namespace std {
typedef signed char int8_t;
typedef short int16_t;
typedef int int32_t;
typedef long long int64_t;
typedef unsigned char uint8_t;
typedef unsigned short uint16_t;
typedef unsigned int uint32_t;
typedef unsigned long long uint64_t;
typedef decltype(sizeof(0)) size_t;
}  // namespace std
#else
#include <cstddef>
#include <cstdint>
#endif

#if defined(__CUDACC__)
#define HK_FI __device__ __forceinline__
#define HK_HD __host__ __device__ __forceinline__
#else
#define HK_FI inline
#define HK_HD inline
#endif

namespace hk {

typedef long long i64;
typedef unsigned long long u64;
typedef int i32;
typedef unsigned int u32;
typedef decltype(sizeof(0)) usize;

// Samples per reduction row: one warp of consecutive samples (hawk/ir/nodes.py:119).
constexpr int kRow = 32;

template <bool B, class T = void> struct enable_if {};
template <class T> struct enable_if<true, T> { typedef T type; };
template <class A, class B> struct is_same { static constexpr bool value = false; };
template <class A> struct is_same<A, A> { static constexpr bool value = true; };
template <class T> struct remove_cvref { typedef T type; };
template <class T> struct remove_cvref<const T> { typedef T type; };
template <class T> struct remove_cvref<T&> { typedef T type; };
template <class T> struct remove_cvref<const T&> { typedef T type; };
template <class T> struct remove_cvref<T&&> { typedef T type; };

}  // namespace hk
