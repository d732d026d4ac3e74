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
// result except with probability ~2^-45 per call; glibc's sin/cos are
// correctly rounded on the same inputs except in rare cases.  Ziv's strategy:
// a cheap evaluation (sincos_fast_parts, error below 2^-65) is rounded when a
// rounding test proves the result (all but ~0.08 % of arguments), else the
// accurate one below runs.  Method of the accurate evaluation:
//   * Cody-Waite reduction x = k*pi/2 + r with pi/2 held as three doubles and
//     every product formed exactly with an FMA (two-product),
//   * Tang's table method on |r| <= pi/4: sin and cos of j/64 from a
//     double-double table, short Taylor series of the remainder |d| <= 1/128
//     (Dekker/Knuth two-sum and two-product for the double-double steps),
//   * one final rounding of the double-double value.
// The coefficients are exact reciprocals of factorials, the table entries
// are sin/cos of exact rationals and pi/2 is computed from Machin's formula
// (gen_sincos_consts.py).  Arguments beyond 2^20 in magnitude are reduced by
// Payne and Hanek's method with the bits of 2/pi (also generated there);
// infinities and NaN give NaN.
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
#else
HK_HD double fma_(double a, double b, double c) { return std::fma(a, b, c); }
HK_HD double rint_(double x) { return std::rint(x); }
HK_HD double fabs_(double x) { return std::fabs(x); }
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

// sin(j/64) and cos(j/64) for j = 0..52 as double-doubles {sin hi, sin lo,
// cos hi, cos lo} (gen_sincos_consts.py: Taylor series of exact rationals).
#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
static __device__ const double __align__(16) kSinCosTableDev[53][4] = {HK_SINCOS_TABLE_DATA};
#endif
#if !defined(__CUDACC_RTC__)
alignas(16) static const double kSinCosTableHost[53][4] = {HK_SINCOS_TABLE_DATA};
#endif

HK_HD void sincos_row(int j, dd* sa, dd* ca) {
#if defined(__CUDA_ARCH__)
    const double2 lo = __ldg(reinterpret_cast<const double2*>(kSinCosTableDev[j]));
    const double2 hi = __ldg(reinterpret_cast<const double2*>(kSinCosTableDev[j]) + 1);
    *sa = dd{lo.x, lo.y};
    *ca = dd{hi.x, hi.y};
#else
    *sa = dd{kSinCosTableHost[j][0], kSinCosTableHost[j][1]};
    *ca = dd{kSinCosTableHost[j][2], kSinCosTableHost[j][3]};
#endif
}

// a * b for double-doubles, unnormalised: |l| may reach a few ulp(h)/2, which
// the sums below absorb (relative error about 2^-104).
HK_HD dd dd_mul_loose(dd a, dd b) {
    const double p = a.h * b.h;
    double e = fma_(a.h, b.h, -p);
    e = fma_(a.h, b.l, e);
    e = fma_(a.l, b.h, e);
    return dd{p, e};
}

// a + b where |b.h| <= |a.h| / 2 (or a.h == 0): no cancellation of the high parts.
HK_HD dd dd_add_small(dd a, dd b) {
    const dd s = fast_two_sum(a.h, b.h);
    return dd{s.h, s.l + (a.l + b.l)};
}

// sin r and cos r of the reduced argument r (|r| <= pi/4 + eps) as
// double-doubles, by Tang's table method: r = a + d with a = j/64 from the
// table and |d| <= 1/128, then
//   sin r = sin a + (sin a (cos d - 1) + cos a sin d),
//   cos r = cos a + (cos a (cos d - 1) - sin a sin d),
//   sin d = d + d z S(z),  cos d - 1 = z C(z),  z = d^2,
// with the Taylor series of S and C cut where the next term is below 2^-100
// of the result.  The three leading coefficients of S and C are carried in
// double-double; the rest, below 2^-19 of the part they are added to, in
// double.  Relative error below 2^-100 (2^-104.5 worst in 2 M arguments
// checked against binary128 sin/cos).
HK_HD void sincos_reduced(dd r, dd* s, dd* c) {
    const double jd = rint_(r.h * 64.0);
    const dd d = fast_two_sum(r.h - jd * 0.015625, r.l);   // r.h - j/64 is exact
    const double ah = fabs_(jd);
    dd sa, ca;
    sincos_row(static_cast<int>(ah), &sa, &ca);
    if (jd < 0.0) sa = dd_neg(sa);
    const dd z = dd_mul_loose(d, d);
    // S(z) = -1/3! + z/5! - z^2/7! + z^3/9! - z^4/11!
    const double s3 = fma_(-inv_fact(11, 0), z.h, inv_fact(9, 0));
    const dd s2 = dd_add_small(fact_inv(7, -1.0), dd{z.h * s3, 0.0});
    const dd s1 = dd_add_small(fact_inv(5, 1.0), dd_mul_loose(z, s2));
    const dd sz = dd_add_small(fact_inv(3, -1.0), dd_mul_loose(z, s1));
    // C(z) = -1/2! + z/4! - z^2/6! + z^3/8! - z^4/10!
    const double c3 = fma_(-inv_fact(10, 0), z.h, inv_fact(8, 0));
    const dd c2 = dd_add_small(fact_inv(6, -1.0), dd{z.h * c3, 0.0});
    const dd c1 = dd_add_small(fact_inv(4, 1.0), dd_mul_loose(z, c2));
    const dd cz = dd_add_small(fact_inv(2, -1.0), dd_mul_loose(z, c1));
    const dd sd = dd_add_small(d, dd_mul_loose(d, dd_mul_loose(z, sz)));   // sin d
    const dd cm = dd_mul_loose(z, cz);                                       // cos d - 1
    const dd ts = dd_add(dd_mul_loose(sa, cm), dd_mul_loose(ca, sd));
    const dd tc = dd_add(dd_mul_loose(ca, cm), dd_neg(dd_mul_loose(sa, sd)));
    *s = dd_add(sa, ts);                     // sa == 0 (j == 0) leaves sd exactly
    *c = dd_add(ca, tc);
}

// The 32-bit words of 2/pi, most significant first.
#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
static __device__ const unsigned kTwoOverPiDev[40] = {HK_TWO_OVER_PI_WORDS};
#endif
#if !defined(__CUDACC_RTC__)
static const unsigned kTwoOverPiHost[40] = {HK_TWO_OVER_PI_WORDS};
#endif

HK_HD unsigned two_over_pi_word(int i) {
#if defined(__CUDA_ARCH__)
    return __ldg(kTwoOverPiDev + i);
#else
    return kTwoOverPiHost[i];
#endif
}

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

HK_HD int clz64(unsigned long long v) {
#if defined(__CUDA_ARCH__)
    return __clzll(static_cast<long long>(v));
#else
    return v ? __builtin_clzll(v) : 64;
#endif
}

HK_HD unsigned long long mul_hi64(unsigned long long a, unsigned long long b) {
#if defined(__CUDA_ARCH__)
    return __umul64hi(a, b);
#else
    return static_cast<unsigned long long>((static_cast<unsigned __int128>(a) * b) >> 64);
#endif
}

// Bits [bit, bit + 64) of the 128-bit lo + hi 2^64 (0 <= bit < 64).
HK_HD unsigned long long funnel64(unsigned long long lo, unsigned long long hi, int bit) {
    return bit ? (lo >> bit) | (hi << (64 - bit)) : lo;
}

// Payne and Hanek's reduction of a finite ax >= 2^20: ax = (4n + q) pi/2 + r
// with |r| <= pi/4, r as a double-double (relative error about 2^-104).
// With ax = m 2^e (m < 2^53), y = ax 2/pi needs only the 8 words of 2/pi
// from i0 = floor((e - 2) / 32): earlier words contribute multiples of 4 and
// later ones less than 2^-165.  P = m * (those 256 bits) is exact in five
// 64-bit limbs; its two bits at the binary point are the quadrant, the 192
// bits below it the fraction, rounded to the nearest quadrant and multiplied
// by pi/2.
HK_HD void reduce_payne_hanek(double ax, int* quadrant, dd* r) {
    typedef unsigned long long u64;
    const u64 b = bits_of(ax);
    const int e = static_cast<int>((b >> 52) & 0x7ff) - 1075;
    const u64 m = (b & ((1ull << 52) - 1ull)) | (1ull << 52);
    const int i0 = e >= 2 ? (e - 2) / 32 : 0;
    u64 p[5];                                       // P, least significant limb first
    u64 carry_hi = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {                   // limb k: words i0 + 7 - 2k (low), i0 + 6 - 2k (high)
        const u64 w = (static_cast<u64>(two_over_pi_word(i0 + 6 - 2 * k)) << 32) |
                      two_over_pi_word(i0 + 7 - 2 * k);
        const u64 lo = m * w;
        const u64 hi = mul_hi64(m, w);              // < 2^53
        const u64 s = lo + carry_hi;
        p[k] = s;
        carry_hi = hi + (s < lo ? 1ull : 0ull);
    }
    p[4] = carry_hi;
    // binary point at bit 32 (i0 + 8) - e, in (222, 288]; take bits [point - 192, point + 2)
    const int sh = 32 * (i0 + 8) - e - 192;         // in (30, 96]
    const bool up = sh >= 64;
    const int bit = sh & 63;
    const u64 f0 = funnel64(up ? p[1] : p[0], up ? p[2] : p[1], bit);
    u64 f1 = funnel64(up ? p[2] : p[1], up ? p[3] : p[2], bit);
    u64 f2 = funnel64(up ? p[3] : p[2], up ? p[4] : p[3], bit);
    const u64 f3 = funnel64(up ? p[4] : p[3], up ? 0ull : p[4], bit);
    int quad = static_cast<int>(f3 & 3ull);
    u64 g0 = f0;
    const bool upper = (f2 >> 63) != 0ull;          // fraction >= 1/2: round up a quadrant
    if (upper) {                                     // |fraction - 1| = 2^192 - F
        quad = (quad + 1) & 3;
        g0 = ~f0 + 1ull;
        f1 = ~f1 + (g0 == 0ull ? 1ull : 0ull);
        f2 = ~f2 + ((g0 == 0ull && f1 == 0ull) ? 1ull : 0ull);
    }
    // normalise (the fraction of a double argument is above 2^-62, so f2 != 0)
    const int lz = clz64(f2);
    const u64 top = lz ? (f2 << lz) | (f1 >> (64 - lz)) : f2;
    const u64 mid = lz ? (f1 << lz) | (g0 >> (64 - lz)) : f1;
    const double scale = from_bits(static_cast<u64>(1023 - 53 - lz) << 52);   // 2^(-53 - lz)
    const double fh = static_cast<double>(top >> 11) * scale;
    const double fl = static_cast<double>(((top & 0x7ffull) << 42) | (mid >> 22)) * scale * 0x1p-53;
    dd f = dd_mul(dd{fh, fl}, dd{kPio2Hi, kPio2Mid});
    if (upper) f = dd_neg(f);
    *quadrant = quad;
    *r = f;
}

// Largest |x| reduced by Cody and Waite's three-part pi/2; beyond it
// reduce_payne_hanek.
constexpr double kCrMax = 1048576.0;   // 2^20

// The rounded sin and cos of r (double-double) in quadrant q.
HK_HD void sincos_quadrant(dd r, int q, double* sx, double* cx) {
    dd s, c;
    sincos_reduced(r, &s, &c);
    const double sr = s.h + s.l;
    const double cr = c.h + c.l;
    const double s1 = (q & 1) ? cr : sr;
    const double c1 = (q & 1) ? sr : cr;
    *sx = (q & 2) ? -s1 : s1;
    *cx = ((q + 1) & 2) ? -c1 : c1;
}

// The cheap first try of Ziv's strategy: sin r and cos r for 2^-27 <= |x| <=
// 2^20 with |r| >= 2^-20, each as h + l with |error| <= 2^-65 |h| (2^-67.3
// worst in 3.8 M arguments against binary128; the error analysis bounds it
// near 2^-66: the d^3 term, about 2^-23.6 of a result >= 2^-7, carries
// three roundings of 2^-53); returns the
// quadrant, or -1 where it does not apply.  The reduction uses pi/2 = C1 + C2
// + C3 with C1 and C2 of 33 bits, so k C1 and k C2 are exact for |k| < 2^20
// and x - k C1 is exact (Sterbenz); the evaluation is the table method of
// sincos_reduced with only the products of the leading terms kept exactly.
HK_HD int sincos_fast_parts(double x, dd* s, dd* c) {
    const double ax = fabs_(x);
    const double kd = rint_(x * kTwoOverPi);
    const double a = x - kd * kPio2C1;                 // both steps exact
    const dd s2 = two_sum(a, -(kd * kPio2C2));         // kd * C2 exact
    const dd r = fast_two_sum(s2.h, s2.l - kd * kPio2C3);
    if (!(ax <= kCrMax) || ax < 0x1p-27 || !(fabs_(r.h) >= 0x1p-20)) return -1;
    const double jd = rint_(r.h * 64.0);
    const double dh = r.h - jd * 0.015625;             // exact
    const double dl = r.l;
    dd sa, ca;
    sincos_row(static_cast<int>(fabs_(jd)), &sa, &ca);
    if (jd < 0.0) sa = dd_neg(sa);
    const double z = dh * dh;
    const double zl = fma_(dh, dh, -z);
    // sin d = dh + sdl;  cos d - 1 = -z/2 + cml
    const double sp = fma_(fma_(fma_(inv_fact(9, 0), z, -inv_fact(7, 0)), z, inv_fact(5, 0)), z, -inv_fact(3, 0));
    const double sdl = fma_(dh * z, sp, dl - dl * z * 0.5);
    const double cp = fma_(fma_(-inv_fact(10, 0), z, inv_fact(8, 0)), z, -inv_fact(6, 0));
    const double cq = fma_(cp, z, inv_fact(4, 0));
    const double cmh = -0.5 * z;
    const double cml = fma_(z * z, cq, -0.5 * zl - dh * dl);
    // sin r = sa + sa (cos d - 1) + ca sin d
    const dd p1 = two_prod(ca.h, dh);
    const dd p2 = two_prod(sa.h, cmh);
    const dd u = fast_two_sum(sa.h, p1.h);             // |sa.h| >= sin(1/64) > |p1.h|, or sa.h == 0
    const dd v = fast_two_sum(u.h, p2.h);
    const double sl = (u.l + v.l) + (p1.l + p2.l) + (sa.l + sa.l * cmh) + (ca.h * sdl + ca.l * dh) + sa.h * cml;
    // cos r = ca + ca (cos d - 1) - sa sin d
    const dd p3 = two_prod(ca.h, cmh);
    const dd p4 = two_prod(sa.h, dh);
    const dd u2 = fast_two_sum(ca.h, p3.h);            // ca.h >= 0.69
    const dd v2 = fast_two_sum(u2.h, -p4.h);
    const double cl = (u2.l + v2.l) + (p3.l - p4.l) + (ca.l + ca.l * cmh) + (ca.h * cml - sa.h * sdl) - sa.l * dh;
    *s = dd{v.h, sl};
    *c = dd{v2.h, cl};
    return static_cast<int>(static_cast<long long>(kd) & 3);
}

// h + l rounded, when every value within 2^-65 |h| of it rounds the same.
HK_HD bool round_sure(dd v, double* out) {
    const double e = 0x1p-65 * fabs_(v.h);
    const double up = v.h + (v.l + e);
    *out = v.h + v.l;
    return up == v.h + (v.l - e) && up == *out;
}

// sin x and cos x, each correctly rounded (see the file comment); arguments
// beyond 2^20, infinities and NaN branch at the end.
HK_HD void sincos_eval(double x, double* sx, double* cx) {
    {
        dd fs, fc;
        const int q = sincos_fast_parts(x, &fs, &fc);
        double sr, cr;
        if (q >= 0 && round_sure(fs, &sr) && round_sure(fc, &cr)) {
            const double s1 = (q & 1) ? cr : sr;
            const double c1 = (q & 1) ? sr : cr;
            *sx = (q & 2) ? -s1 : s1;
            *cx = ((q + 1) & 2) ? -c1 : c1;
            return;
        }
    }
    const double ax = fabs_(x);
    const bool in_range = ax <= kCrMax;      // false for NaN and infinities
    const double xr = in_range ? x : 0.0;
    const double kd = rint_(xr * kTwoOverPi);
    const dd p = two_prod(kd, kPio2Hi);
    const double a = xr - p.h;               // exact: x and p.h are within a factor 2 (or kd == 0)
    dd r = two_sum(a, -p.l);
    r = dd_add_accurate(r, dd_neg(two_prod(kd, kPio2Mid)));
    r = dd_add_accurate(r, dd{-kd * kPio2Lo, 0.0});
    double so, co;
    sincos_quadrant(r, static_cast<int>(static_cast<long long>(kd) & 3), &so, &co);
    const bool tiny = ax < 0x1p-27;          // sin x = x, cos x = 1 after rounding
    so = tiny ? x : so;
    co = tiny ? 1.0 : co;
    if (!in_range) {
        if (ax - ax == 0.0) {                // finite: Payne-Hanek, then the sign of x
            int q;
            dd rr;
            reduce_payne_hanek(ax, &q, &rr);
            if (x < 0.0) {
                q = (4 - q) & 3;
                rr = dd_neg(rr);
            }
            sincos_quadrant(rr, q, &so, &co);
        } else {                             // NaN and infinities: NaN
            so = x - x;
            co = x - x;
        }
    }
    *sx = so;
    *cx = co;
}

struct SinCos {
    double s, c;
};

// The one evaluation of sincos_eval for an argument, out of line and marked
// pure (it reads only the constant tables): a body that takes sin and cos of
// the same argument calls it once (the compiler merges calls with equal
// arguments), and the Payne-Hanek branch does not add to the registers of the
// calling kernel.
#if defined(__CUDA_ARCH__)
__device__ __noinline__ __attribute__((pure)) SinCos sincos_pure(double x) {
    SinCos r;
    sincos_eval(x, &r.s, &r.c);
    return r;
}
#else
inline SinCos sincos_pure(double x) {
    SinCos r;
    sincos_eval(x, &r.s, &r.c);
    return r;
}
#endif

HK_HD void sincos_cr(double x, double* sx, double* cx) {
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
