// The device library's sin/cos (hk/math.cuh), compiled for the host, against
// the host's glibc sin/cos: arguments drawn over every range of glibc's method
// (the Taylor range, the table range, pi/2 - |x|, the four-part reduction and
// the large-argument reduction) and the special values.  Prints the mismatch
// count; exits non-zero if any argument differs in any bit.
//
//   g++ -O2 -std=c++17 -ffp-contract=off -I<hk include root> sincos_libm_check.cpp
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "hk/math.cuh"

static std::uint64_t state = 88172645463325252ull;

static std::uint64_t next() {
    state ^= state << 13;
    state ^= state >> 7;
    state ^= state << 17;
    return state;
}

static double uniform(double lo, double hi) { return lo + (hi - lo) * ((next() >> 11) * 0x1p-53); }

static bool same(double a, double b) {
    return std::memcmp(&a, &b, sizeof a) == 0 || (std::isnan(a) && std::isnan(b));
}

int main(int argc, char** argv) {
    const long n = argc > 1 ? std::atol(argv[1]) : 200000;
    // called through pointers so that the compiler neither folds nor merges them
    double (*volatile libm_sin)(double) = ::sin;
    double (*volatile libm_cos)(double) = ::cos;
    const double ranges[][2] = {{1e-9, 0.126},  {0.126, 0.855},       {0.855, 2.426},     {2.426, 7.0},
                                {7.0, 1e4},     {1e4, 105414350.0},   {105414350.0, 1e9}, {1e9, 1e300}};
    long bad = 0, total = 0;
    for (int r = 0; r < 8; ++r) {
        for (long i = 0; i < n; ++i) {
            double x = r < 6 ? uniform(ranges[r][0], ranges[r][1])
                             : std::exp(uniform(std::log(ranges[r][0]), std::log(ranges[r][1])));
            if (next() & 1) x = -x;
            double s, c;
            hk::math::sincos(x, &s, &c);
            ++total;
            if (!same(s, libm_sin(x)) || !same(c, libm_cos(x))) {
                if (bad < 5) std::printf("x = %a: sin %a (libm %a), cos %a (libm %a)\n", x, s, libm_sin(x), c, libm_cos(x));
                ++bad;
            }
        }
    }
    const double special[] = {0.0, -0.0, 0x1p-1074, 0x1p-30, -0x1p-27, 0x1p-26, 0.126, 0.85546875, 2.426265,
                              105414350.0, 1e22, 6381956970095103.0 * 0x1p797, 1.7976931348623157e308,
                              INFINITY, -INFINITY, NAN};
    for (double x : special) {
        double s, c;
        hk::math::sincos(x, &s, &c);
        ++total;
        if (!same(s, libm_sin(x)) || !same(c, libm_cos(x))) {
            std::printf("x = %a: sin %a (libm %a), cos %a (libm %a)\n", x, s, libm_sin(x), c, libm_cos(x));
            ++bad;
        }
    }
    std::printf("mismatches %ld of %ld\n", bad, total);
    return bad != 0;
}
