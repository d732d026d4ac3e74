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
// the host's libm can change an integer result.  They are therefore computed
// here by glibc's own method, operation for operation, so that every result
// has glibc's bits: the dbl-64 sin/cos of glibc 2.39
// (sysdeps/ieee754/dbl-64/s_sin.c, branred.c; coefficients in s_sin.c and
// usncs.h) as its x86-64 multiarch build runs them on a host with FMA (the
// build GCC compiles with -mfma -mavx2: every multiply whose only use is an
// add or subtract is fused, a multiply with two uses is not).  The method:
//   * |x| < 0.855: sin and cos of x directly;  |x| < 2.426: sin x = cos(pi/2
//     - |x|) and cos x = sin(pi/2 - |x|) with pi/2 = hp0 + hp1;  |x| <
//     105414350: x = n pi/2 + (a + da) by a four-part pi/2 (mp1, mp2, pp3,
//     pp4);  beyond: the 24-bit chunks of 2/pi (branred);
//   * sin/cos of a + da: |a| rounded to a multiple of 1/128 (adding 1.5 2^45),
//     sin and cos of that node from a double-double table, the remainder's
//     sin/cos by short polynomials, combined with the table's low parts;
//     |a| < 0.126 in sin: a Taylor-like polynomial of a alone.
// The polynomial coefficients are glibc's published values (they are fitted,
// not a function of pi); the table, the splits of pi/2 and the chunks of 2/pi
// are mathematics and are generated exactly (gen_sincos_consts.py).
// Results differ from glibc's build WITHOUT FMA (its SSE2 variant, on hosts
// lacking FMA) in about 0.1 % of arguments by one ulp.
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
HK_HD double fabs_(double x) { return ::fabs(x); }
HK_HD double copysign_(double x, double y) { return ::copysign(x, y); }
#else
HK_HD double fma_(double a, double b, double c) { return std::fma(a, b, c); }
HK_HD double fabs_(double x) { return std::fabs(x); }
HK_HD double copysign_(double x, double y) { return std::copysign(x, y); }
#endif

HK_HD unsigned long long bits_of(double x) {
#if defined(__CUDA_ARCH__)
    return static_cast<unsigned long long>(__double_as_longlong(x));
#else
    unsigned long long b;
    __builtin_memcpy(&b, &x, sizeof b);
    return b;
#endif
}

HK_HD double from_bits(unsigned long long b) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double(static_cast<long long>(b));
#else
    double x;
    __builtin_memcpy(&x, &b, sizeof x);
    return x;
#endif
}

// glibc's coefficients: sin d ~ d + sn3 d^3 + sn5 d^5, cos d ~ 1 - (cs2 d^2 +
// cs4 d^4 + cs6 d^6) around a table node; s1..s5 for sin of |x| < 0.126.
constexpr double kSn3 = -0x1.5555555555515p-3;
constexpr double kSn5 = 0x1.11110e829872fp-7;
constexpr double kCs2 = 0x1.0000000000000p-1;
constexpr double kCs4 = -0x1.5555555555535p-5;
constexpr double kCs6 = 0x1.6c16bedd9e239p-10;
constexpr double kS1 = -0x1.5555555555555p-3;
constexpr double kS2 = 0x1.1111111110ecep-7;
constexpr double kS3 = -0x1.a01a019db08b8p-13;
constexpr double kS4 = 0x1.71de27b9a7ed9p-19;
constexpr double kS5 = -0x1.addffc2fcdf59p-26;
constexpr double kBig = 0x1.8p45;      // ulp 2^-7: big + |x| rounds |x| to a multiple of 1/128
constexpr double kToInt = 0x1.8p52;    // ulp 1: t + toInt rounds t to an integer
constexpr double kBig52 = 0x1.8p52;
constexpr double kBig54 = 0x1.8p54;
constexpr double kSplit = 134217729.0; // 2^27 + 1 (Dekker's split)
constexpr int kTableLast = 109;        // |x| < 0.85546875 rounds to node <= 109/128

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
static __device__ const double __align__(16) kSinCos128Dev[110][4] = {HK_SINCOS128_TABLE_DATA};
static __device__ const double kTwoOverPi24Dev[75] = {HK_TWO_OVER_PI_24};
#endif
#if !defined(__CUDACC_RTC__)
alignas(16) static const double kSinCos128Host[110][4] = {HK_SINCOS128_TABLE_DATA};
static const double kTwoOverPi24Host[75] = {HK_TWO_OVER_PI_24};
#endif

struct Node {
    double sn, ssn, cs, ccs;     // sin(k/128) = sn + ssn, cos(k/128) = cs + ccs
};

// The table node of u = big + |x| (its low word is round(128 |x|)); the
// index is held inside the table so that no argument can read past it.
HK_HD Node node_of(double u) {
    unsigned k = static_cast<unsigned>(bits_of(u));
    k = k < kTableLast ? k : kTableLast;
#if defined(__CUDA_ARCH__)
    const double2 s = __ldg(reinterpret_cast<const double2*>(kSinCos128Dev[k]));
    const double2 c = __ldg(reinterpret_cast<const double2*>(kSinCos128Dev[k]) + 1);
    return Node{s.x, s.y, c.x, c.y};
#else
    return Node{kSinCos128Host[k][0], kSinCos128Host[k][1], kSinCos128Host[k][2], kSinCos128Host[k][3]};
#endif
}

HK_HD double two_over_pi_24(int i) {
#if defined(__CUDA_ARCH__)
    return __ldg(kTwoOverPi24Dev + i);
#else
    return kTwoOverPi24Host[i];
#endif
}

// sin(x + dx) for |x| < 0.855 (glibc's do_sin).
HK_HD double do_sin(double x, double dx) {
    const double xold = x;
    if (fabs_(x) < 0.126) {
        const double xx = x * x;
        double q = fma_(kS5, xx, kS4);
        q = fma_(q, xx, kS3);
        q = fma_(q, xx, kS2);
        q = fma_(q, xx, kS1);
        const double t = fma_(fma_(q, x, -(0.5 * dx)), xx, dx);
        return x + t;
    }
    if (x <= 0) dx = -dx;
    const double u = kBig + fabs_(x);
    x = fabs_(x) - (u - kBig);
    const Node n = node_of(u);
    const double xx = x * x;
    const double s = x + fma_(x * xx, fma_(xx, kSn5, kSn3), dx);
    const double c = fma_(x, dx, xx * fma_(xx, fma_(xx, kCs6, kCs4), kCs2));
    double cor = fma_(s, n.ccs, n.ssn);
    cor = fma_(-n.sn, c, cor);
    cor = fma_(n.cs, s, cor);
    return copysign_(n.sn + cor, xold);
}

// cos(x + dx) for |x| < 0.855 (glibc's do_cos).
HK_HD double do_cos(double x, double dx) {
    if (x < 0) dx = -dx;
    const double u = kBig + fabs_(x);
    x = fabs_(x) - (u - kBig) + dx;
    const Node n = node_of(u);
    const double xx = x * x;
    const double s = fma_(x * xx, fma_(xx, kSn5, kSn3), x);
    const double c = xx * fma_(xx, fma_(xx, kCs6, kCs4), kCs2);
    double cor = fma_(-s, n.ssn, n.ccs);
    cor = fma_(-n.cs, c, cor);
    cor = fma_(-n.sn, s, cor);
    return n.cs + cor;
}

// x = n pi/2 + (a + da) for |x| < 105414350; returns n mod 4 (reduce_sincos).
HK_HD int reduce_sincos(double x, double* a, double* da) {
    const double t = fma_(x, kHpInv, kToInt);
    const double xn = t - kToInt;
    const int n = static_cast<int>(bits_of(t) & 3);
    double y = fma_(-xn, kMp1, x);
    y = fma_(-xn, kMp2, y);
    double t1 = xn * kPp3;
    const double t2 = y - t1;
    double db = (y - t2) - t1;
    t1 = xn * kPp4;
    const double b = t2 - t1;
    db += (t2 - b) - t1;
    *a = b;
    *da = db;
    return n;
}

// One half of branred: the product of x1 (at most 27 significant bits) with
// the chunks of 2/pi that reach its binary point, as an integer part mod 4
// (sum) and a fraction b + bb.
HK_HD void branred_half(double x1, double* sum_o, double* b_o, double* bb_o) {
    double r[6];
    int k = static_cast<int>((bits_of(x1) >> 52) & 2047);
    k = (k - 450) / 24;
    if (k < 0) k = 0;
    double gor = from_bits(bits_of(0x1p576) - (static_cast<unsigned long long>(k * 24) << 52));
    for (int i = 0; i < 6; ++i) {
        r[i] = x1 * two_over_pi_24(k + i) * gor;
        gor *= 0x1p-24;
    }
    double sum = 0.0, s;
    for (int i = 0; i < 3; ++i) {
        s = (r[i] + kBig52) - kBig52;
        sum += s;
        r[i] -= s;
    }
    double t = 0.0;
    for (int i = 0; i < 6; ++i) t += r[5 - i];
    double bb = (((((r[0] - t) + r[1]) + r[2]) + r[3]) + r[4]) + r[5];
    s = (t + kBig52) - kBig52;
    sum += s;
    t -= s;
    const double b = t + bb;
    bb = (t - b) + bb;
    s = (sum + kBig54) - kBig54;
    sum -= s;
    *sum_o = sum;
    *b_o = b;
    *bb_o = bb;
}

// x = n pi/2 + (a + da) for 105414350 <= |x| < 2^1024 (glibc's branred:
// x split into two halves of 26 and 27 bits, each multiplied by the 24-bit
// chunks of 2/pi, the fractions combined, times pi/2 in double-double).
HK_HD int branred(double x, double* a, double* da) {
    x *= 0x1p-600;
    double t = x * kSplit;
    const double x1 = t - (t - x);
    const double x2 = x - x1;
    double sum1, b1, bb1, sum2, b2, bb2;
    branred_half(x1, &sum1, &b1, &bb1);
    branred_half(x2, &sum2, &b2, &bb2);
    double sum = sum1 + sum2;
    double b = b1 + b2;
    double bb = (fabs_(b1) > fabs_(b2)) ? (b1 - b) + b2 : (b2 - b) + b1;
    if (b > 0.5) {
        b -= 1.0;
        sum += 1.0;
    } else if (b < -0.5) {
        b += 1.0;
        sum -= 1.0;
    }
    double s = b + (bb + bb1 + bb2);
    t = ((b - s) + bb) + (bb1 + bb2);
    b = s * kSplit;
    const double t1 = b - (b - s);
    const double t2 = s - t1;
    b = s * kHp0;
    bb = (((t1 * kMp1 - b) + t1 * kBrMp2) + t2 * kMp1) + (t2 * kBrMp2 + s * kHp1 + t * kHp0);
    s = b + bb;
    t = (b - s) + bb;
    *a = s;
    *da = t;
    return static_cast<int>(sum) & 3;
}

struct SinCos {
    double s, c;
};

struct Reduced {
    double a, da;
    int n;
};

// branred out of line, its result returned by value: the large-argument path
// adds neither registers nor stack to the callers of the common path.
#if defined(__CUDA_ARCH__)
__device__ __noinline__ Reduced branred_call(double x) {
#else
inline Reduced branred_call(double x) {
#endif
    Reduced r;
    r.n = branred(x, &r.a, &r.da);
    return r;
}

// sin x and cos x with glibc's bits.  Each range's argument for glibc's
// do_sin and for its do_cos is chosen first, so every call evaluates one
// do_sin and one do_cos whatever the range (a warp whose lanes fall in
// different ranges does not run each range's evaluation in turn):
//   |x| < 0.855:       sin = do_sin(x, 0),                  cos = do_cos(x, 0)
//   |x| < 2.426:       sin = copysign(do_cos(hp0 - |x|, hp1), x),
//                      cos = do_sin(a, da), a + da = (hp0 - |x|) + hp1
//   otherwise:         x = n pi/2 + (a + da); sin and cos are do_sin(a, da) and
//                      do_cos(a, da) in the order and with the signs of
//                      quadrant n (cos: quadrant n + 1);
// tiny arguments return x (sin, |x| < 2^-26) and 1 (cos, |x| < 2^-27), and
// infinities and NaN give NaN.
HK_HD SinCos sincos_eval(double x) {
    const unsigned hi = static_cast<unsigned>(bits_of(x) >> 32) & 0x7fffffffu;
    const double ax = fabs_(x);
    double ra, rda;
    int n = 0;
    if (hi >= 0x419921fbu) {
        if (hi < 0x7ff00000u) {
            const Reduced red = branred_call(x);
            ra = red.a;
            rda = red.da;
            n = red.n;
        } else {
            ra = 0.0;
            rda = 0.0;
        }
    } else {
        n = reduce_sincos(x, &ra, &rda);
    }
    const double y = kHp0 - ax;
    const double ya = y + kHp1;
    const double yda = (y - ya) + kHp1;
    const bool low = hi < 0x3feb6000u;
    const bool mid = !low && hi < 0x400368fdu;
    const double sa = low ? x : (mid ? ya : ra);
    const double sda = low ? 0.0 : (mid ? yda : rda);
    const double ca = low ? x : (mid ? y : ra);
    const double cda = low ? 0.0 : (mid ? kHp1 : rda);
    const double S = do_sin(sa, sda);
    const double C = do_cos(ca, cda);
    SinCos r;
    if (low) {
        r.s = hi < 0x3e500000u ? x : S;
        r.c = hi < 0x3e400000u ? 1.0 : C;
    } else if (mid) {
        r.s = copysign_(C, x);
        r.c = S;
    } else {
        const double q0 = (n & 1) ? C : S;
        const double q1 = (n & 1) ? S : C;
        r.s = (n & 2) ? -q0 : q0;
        r.c = ((n + 1) & 2) ? -q1 : q1;
        if (hi >= 0x7ff00000u) r.s = r.c = x - x;
    }
    return r;
}

// The one evaluation of sincos_eval for an argument, out of line and marked
// pure (it reads only the constant tables): a body that takes sin and cos of
// the same argument calls it once (the compiler merges calls with equal
// arguments), and the large-argument branch does not add to the registers of
// the calling kernel.
#if defined(__CUDA_ARCH__)
__device__ __noinline__ __attribute__((pure)) SinCos sincos_pure(double x) { return sincos_eval(x); }
#else
inline SinCos sincos_pure(double x) { return sincos_eval(x); }
#endif

HK_HD void sincos_libm(double x, double* sx, double* cx) {
    const SinCos r = sincos_pure(x);
    *sx = r.s;
    *cx = r.c;
}

}  // namespace detail

namespace math {

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
#define HK_MATH HK_FI
#else
#define HK_MATH inline
#endif

HK_MATH double sin(double x) { double s, c; detail::sincos_libm(x, &s, &c); return s; }
HK_MATH double cos(double x) { double s, c; detail::sincos_libm(x, &s, &c); return c; }
HK_MATH void sincos(double x, double* s, double* c) { detail::sincos_libm(x, s, c); }
HK_MATH float sin(float x) { double s, c; detail::sincos_libm(static_cast<double>(x), &s, &c); return static_cast<float>(s); }
HK_MATH float cos(float x) { double s, c; detail::sincos_libm(static_cast<double>(x), &s, &c); return static_cast<float>(c); }
HK_MATH void sincos(float x, float* s, float* c) {
    double sd, cd;
    detail::sincos_libm(static_cast<double>(x), &sd, &cd);
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
