// hawk_b200 device library: scalar math for the per-sample body.
//
// The body text names ``<ns>::math::<fn>`` for every rank-0 transcendental
// (the op tables at hawk/emit/spelling.py:81-99).  The reference's host target
// resolves those to glibc's libm; its serial oracle is compared bit for bit
// on integer planes (hawk/compile/toolchain.py:897-900 builds the host with
// -ffp-contract=off, tests/test_math_parity.py:4-14 pins host == glibc).
//
// sin and cos decide data-dependent control flow in loop kernels (a Newton
// iteration count is an int32 output plane), so a last-bit difference from
// glibc can change an integer result.  They are therefore computed here to
// double-double accuracy and rounded once, which gives the correctly rounded
// result except with probability ~2^-40 per call; glibc's sin/cos are
// correctly rounded on the same inputs except in rare cases.  Method:
//   * Cody-Waite reduction x = k*pi/2 + r with pi/2 held as three doubles and
//     every product formed exactly with an FMA (two-product),
//   * the Taylor series of sin r and cos r, |r| <= pi/4, whose terms above
//     r^13 (sin) / r^14 (cos) are summed in double and the rest in
//     double-double (Dekker/Knuth two-sum and two-product),
//   * one final rounding of the double-double value.
// The coefficients are exact reciprocals of factorials and pi/2 is computed
// from Machin's formula (gen_sincos_consts.py).  Arguments beyond 2^20 in
// magnitude, infinities and NaN take the platform's sin/cos.
//
// Every other function calls the CUDA math library directly.
#pragma once
#include "base.cuh"
#include "sincos_consts.cuh"

#if !defined(__CUDACC_RTC__)
#include <cmath>
#endif

namespace hk {
namespace detail {

#if defined(__CUDA_ARCH__)
HK_HD double fma_(double a, double b, double c) { return __fma_rn(a, b, c); }
HK_HD double rint_(double x) { return ::rint(x); }
HK_HD double fabs_(double x) { return ::fabs(x); }
HK_HD double libm_sin(double x) { return ::sin(x); }
HK_HD double libm_cos(double x) { return ::cos(x); }
#else
HK_HD double fma_(double a, double b, double c) { return std::fma(a, b, c); }
HK_HD double rint_(double x) { return std::rint(x); }
HK_HD double fabs_(double x) { return std::fabs(x); }
HK_HD double libm_sin(double x) { return std::sin(x); }
HK_HD double libm_cos(double x) { return std::cos(x); }
#endif

// An unevaluated sum h + l with |l| <= ulp(h) / 2.
struct dd {
    double h, l;
};

// Knuth's two-sum: s + e == a + b exactly.
HK_HD dd two_sum(double a, double b) {
    const double s = a + b;
    const double bb = s - a;
    const double e = (a - (s - bb)) + (b - bb);
    return dd{s, e};
}

// Dekker's fast two-sum, valid when |a| >= |b| (or a == 0).
HK_HD dd fast_two_sum(double a, double b) {
    const double s = a + b;
    const double e = b - (s - a);
    return dd{s, e};
}

// The exact product a * b as a double-double (one FMA).
HK_HD dd two_prod(double a, double b) {
    const double p = a * b;
    return dd{p, fma_(a, b, -p)};
}

HK_HD dd dd_mul(dd a, dd b) {
    const double p = a.h * b.h;
    double e = fma_(a.h, b.h, -p);
    e = fma_(a.h, b.l, e);
    e = fma_(a.l, b.h, e);
    return fast_two_sum(p, e);
}

// Sum of two double-doubles whose high parts do not cancel catastrophically
// (true of every Horner step below: each partial is dominated by its constant).
HK_HD dd dd_add(dd a, dd b) {
    const dd s = two_sum(a.h, b.h);
    return fast_two_sum(s.h, (s.l + a.l) + b.l);
}

// Sum of two double-doubles, accurate under cancellation (argument reduction).
HK_HD dd dd_add_accurate(dd a, dd b) {
    dd s = two_sum(a.h, b.h);
    const dd t = two_sum(a.l, b.l);
    s = fast_two_sum(s.h, s.l + t.h);
    return fast_two_sum(s.h, s.l + t.l);
}

HK_HD dd dd_neg(dd a) { return dd{-a.h, -a.l}; }

HK_HD dd fact_inv(int n, double sign) {
    return dd{sign * inv_fact(n, 0), sign * inv_fact(n, 1)};
}

// sin r and cos r of the reduced argument r (|r| <= pi/4 + eps), both as
// double-doubles; z = r*r is shared.
HK_HD void sincos_reduced(dd r, dd* s, dd* c) {
    const dd z = dd_mul(r, r);
    // sin: r * sum_{n=0..13} (-1)^n z^n / (2n+1)!.  Terms n >= 7 (below 2^-45
    // of the result) are summed in double, the rest in double-double.
    double ts = -inv_fact(27, 0);
#pragma unroll
    for (int n = 12; n >= 7; --n)
        ts = fma_(ts, z.h, ((n & 1) ? -1.0 : 1.0) * inv_fact(2 * n + 1, 0));
    dd ps = two_prod(ts, z.h);
#pragma unroll
    for (int n = 6; n >= 0; --n) {
        ps = dd_add(ps, fact_inv(2 * n + 1, (n & 1) ? -1.0 : 1.0));
        if (n > 0) ps = dd_mul(ps, z);
    }
    *s = dd_mul(ps, r);
    // cos: sum_{n=0..14} (-1)^n z^n / (2n)!.  Terms n >= 8 in double.
    double tc = inv_fact(28, 0);
#pragma unroll
    for (int n = 13; n >= 8; --n)
        tc = fma_(tc, z.h, ((n & 1) ? -1.0 : 1.0) * inv_fact(2 * n, 0));
    dd pc = two_prod(tc, z.h);
#pragma unroll
    for (int n = 7; n >= 0; --n) {
        pc = dd_add(pc, fact_inv(2 * n, (n & 1) ? -1.0 : 1.0));
        if (n > 0) pc = dd_mul(pc, z);
    }
    *c = pc;
}

// Largest |x| reduced here; beyond it the platform's functions are used.
constexpr double kCrMax = 1048576.0;   // 2^20

// sin x and cos x, each correctly rounded (see the file comment).
HK_HD void sincos_cr(double x, double* sx, double* cx) {
    const double ax = fabs_(x);
    if (!(ax <= kCrMax)) {                 // NaN, infinities, huge arguments
        *sx = libm_sin(x);
        *cx = libm_cos(x);
        return;
    }
    if (ax < 0x1p-27) {                    // sin x = x, cos x = 1 after rounding
        *sx = x;
        *cx = 1.0;
        return;
    }
    const double kd = rint_(x * kTwoOverPi);
    dd r;
    if (kd == 0.0) {
        r = dd{x, 0.0};
    } else {
        const dd p = two_prod(kd, kPio2Hi);
        const double a = x - p.h;          // exact: x and p.h are within a factor 2
        r = two_sum(a, -p.l);
        r = dd_add_accurate(r, dd_neg(two_prod(kd, kPio2Mid)));
        r = dd_add_accurate(r, dd{-kd * kPio2Lo, 0.0});
    }
    dd s, c;
    sincos_reduced(r, &s, &c);
    const long long q = static_cast<long long>(kd) & 3;
    const double sr = s.h + s.l;
    const double cr = c.h + c.l;
    switch (q) {
        case 0: *sx = sr; *cx = cr; break;
        case 1: *sx = cr; *cx = -sr; break;
        case 2: *sx = -sr; *cx = -cr; break;
        default: *sx = -cr; *cx = sr; break;
    }
}

}  // namespace detail

namespace math {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
#define HK_MATH HK_FI
#else
#define HK_MATH inline
#endif

HK_MATH double sin(double x) { double s, c; detail::sincos_cr(x, &s, &c); return s; }
HK_MATH double cos(double x) { double s, c; detail::sincos_cr(x, &s, &c); return c; }
HK_MATH void sincos(double x, double* s, double* c) { detail::sincos_cr(x, s, c); }
HK_MATH float sin(float x) { double s, c; detail::sincos_cr(static_cast<double>(x), &s, &c); return static_cast<float>(s); }
HK_MATH float cos(float x) { double s, c; detail::sincos_cr(static_cast<double>(x), &s, &c); return static_cast<float>(c); }
HK_MATH void sincos(float x, float* s, float* c) {
    double sd, cd;
    detail::sincos_cr(static_cast<double>(x), &sd, &cd);
    *s = static_cast<float>(sd);
    *c = static_cast<float>(cd);
}

#if defined(__CUDA_ARCH__)
#define HK_UNARY(NAME, DFN, FFN) \
    HK_MATH double NAME(double x) { return ::DFN(x); } \
    HK_MATH float NAME(float x) { return ::FFN(x); }
#define HK_BINARY(NAME, DFN, FFN) \
    HK_MATH double NAME(double x, double y) { return ::DFN(x, y); } \
    HK_MATH float NAME(float x, float y) { return ::FFN(x, y); }
#else
#define HK_UNARY(NAME, DFN, FFN) \
    HK_MATH double NAME(double x) { return std::DFN(x); } \
    HK_MATH float NAME(float x) { return std::DFN(x); }
#define HK_BINARY(NAME, DFN, FFN) \
    HK_MATH double NAME(double x, double y) { return std::DFN(x, y); } \
    HK_MATH float NAME(float x, float y) { return std::DFN(x, y); }
#endif

HK_UNARY(abs, fabs, fabsf)
HK_UNARY(sqrt, sqrt, sqrtf)
HK_UNARY(exp, exp, expf)
HK_UNARY(log, log, logf)
HK_UNARY(tan, tan, tanf)
HK_UNARY(tanh, tanh, tanhf)
HK_UNARY(asin, asin, asinf)
HK_UNARY(acos, acos, acosf)
HK_UNARY(atan, atan, atanf)
HK_UNARY(floor, floor, floorf)
HK_UNARY(exp2, exp2, exp2f)
HK_UNARY(expm1, expm1, expm1f)
HK_UNARY(log2, log2, log2f)
HK_UNARY(log10, log10, log10f)
HK_UNARY(log1p, log1p, log1pf)
HK_UNARY(cbrt, cbrt, cbrtf)
HK_UNARY(sinh, sinh, sinhf)
HK_UNARY(cosh, cosh, coshf)
HK_UNARY(asinh, asinh, asinhf)
HK_UNARY(acosh, acosh, acoshf)
HK_UNARY(atanh, atanh, atanhf)
HK_UNARY(ceil, ceil, ceilf)
HK_UNARY(trunc, trunc, truncf)
HK_UNARY(round, round, roundf)
HK_UNARY(rint, rint, rintf)
HK_UNARY(erf, erf, erff)
HK_UNARY(erfc, erfc, erfcf)
HK_BINARY(pow, pow, powf)
HK_BINARY(fmin, fmin, fminf)
HK_BINARY(fmax, fmax, fmaxf)
HK_BINARY(atan2, atan2, atan2f)
HK_BINARY(hypot, hypot, hypotf)
HK_BINARY(copysign, copysign, copysignf)
HK_BINARY(fmod, fmod, fmodf)
HK_BINARY(remainder, remainder, remainderf)
HK_BINARY(fdim, fdim, fdimf)
#undef HK_UNARY
#undef HK_BINARY

// 1/sqrt(x) with both operations correctly rounded (a host twin exists in libm terms).
HK_MATH double rsqrt(double x) { return 1.0 / sqrt(x); }
HK_MATH float rsqrt(float x) { return 1.0f / sqrt(x); }

template <class T> HK_MATH bool isnan(T x) { return x != x; }
template <class T> HK_MATH bool isinf(T x) { return x == x && (x - x) != (x - x); }
template <class T> HK_MATH bool isfinite(T x) { return (x - x) == (x - x); }

HK_MATH double fma(double a, double b, double c) { return detail::fma_(a, b, c); }
HK_MATH float fma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return std::fma(a, b, c);
#endif
}

// clip(x, lo, hi): x held inside [lo, hi], NaN bounds ignored as fmin/fmax do.
template <class T> HK_MATH T clip(T x, T lo, T hi) { return fmin(fmax(x, lo), hi); }

// sign(x): -1, 0 or +1 (a NaN stays NaN, a zero keeps its sign).
template <class T> HK_MATH T sign(T x) {
    if (x > T(0)) return T(1);
    if (x < T(0)) return T(-1);
    return x;
}

}  // namespace math
}  // namespace hk
