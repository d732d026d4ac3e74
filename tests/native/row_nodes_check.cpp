// The device library's row nodes (hk/sample_sum.cuh), compiled for the host,
// against the row the reference's node rule makes: a 32-sample row is a tree
// with lanes paired across bit 4, then 3, ..., 0; each node is
//     t = s + s2;  c = finite(t) ? (c + c2) + err : 0;  s = t
// with err the ordered Fast2Sum residual, larger magnitude first, +0 for a
// zero residual (hawk/_cells.py:44-49).  The device joins the first level with
// the residual alone (every compensation is still zero), every later node
// with pair_combine_unchecked (Knuth's 2Sum residual with no + 0 and no
// finiteness test), either operand first (the butterfly's two lanes of a pair
// compute the same node from opposite sides), and settles the root with
// root_comp.  Rows are drawn to hit zero residuals, exact cancellations,
// signed zeros (whole rows of them too), tiny and huge values and non-finite
// samples.
// Prints the mismatch count; exits non-zero if any row differs in any bit.
//
//   g++ -O2 -std=c++17 -ffp-contract=off -I<hk include root> row_nodes_check.cpp
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "hk/sample_sum.cuh"

static std::uint64_t state = 0x9E3779B97F4A7C15ull;

static std::uint64_t next() {
    state ^= state << 13;
    state ^= state >> 7;
    state ^= state << 17;
    return state;
}

static double uniform() { return (next() >> 11) * 0x1p-53; }

static bool same(double a, double b) {
    return std::memcmp(&a, &b, sizeof a) == 0 || (std::isnan(a) && std::isnan(b));
}

static double sample(int kind, double base) {
    switch (kind) {
        case 0: return (uniform() - 0.5) * 8.0;
        case 1: return std::ldexp(uniform() - 0.5, static_cast<int>(next() % 200) - 100);
        case 2: return (next() & 1) ? 0.0 : -0.0;
        case 3: return (next() & 1) ? base : -base;                 // cancels another sample exactly
        case 4: return std::ldexp(1.0, static_cast<int>(next() % 60) - 30) * ((next() & 1) ? 1 : -1);
        case 5: return std::ldexp(uniform(), 1000);                 // overflows some sums
        default: return (next() % 64 == 0) ? NAN : (uniform() - 0.5);
    }
}

// The reference's node, as the rule above states it.
static void reference_node(double& s, double& c, double s2, double c2) {
    const double t = s + s2;
    const bool first_big = std::fabs(s) >= std::fabs(s2);
    const double big = first_big ? s : s2, small = first_big ? s2 : s;
    const double err = (small - (t - big)) + 0.0;
    c = hk::ss::finite(t) ? (c + c2) + err : 0.0;
    s = t;
}

int main(int argc, char** argv) {
    const long rows = argc > 1 ? std::atol(argv[1]) : 100000;
    long bad = 0;
    // the residual is never -0, so it needs no + 0 (every pair of these values,
    // both signs, and the exact cancellations among them)
    const double mags[] = {0.0, 0x1p-1074, 0x1p-1022, 0x1.8p-60, 1.0, 1.5, 0x1.fffffffffffffp0, 0x1p52, 0x1p1023};
    for (double ma : mags)
        for (double mb : mags)
            for (int sg = 0; sg < 4; ++sg) {
                const double a = (sg & 1) ? -ma : ma, b = (sg & 2) ? -mb : mb;
                const double t = a + b;
                const double e = hk::ss::two_sum_err(a, b, t);
                if (hk::ss::finite(t) && e == 0.0 && std::signbit(e)) {
                    std::printf("residual of %a + %a is -0\n", a, b);
                    ++bad;
                }
            }
    for (long r = 0; r < rows; ++r) {
        const int mix = static_cast<int>(next() % 7);
        double x[32];
        const double base = (uniform() - 0.5) * 4.0;
        for (int l = 0; l < 32; ++l) x[l] = sample((next() % 3 == 0) ? mix : static_cast<int>(next() % 5), base);
        if (r % 16 == 0)
            for (int l = 0; l < 32; ++l) x[l] = sample(2, base);
        if (r % 16 == 1)
            for (int l = 0; l < 32; ++l) x[l] = (l < 16) ? sample(3, base) : -x[l - 16];

        double rs[32], rc[32];
        for (int l = 0; l < 32; ++l) rs[l] = x[l], rc[l] = 0.0;
        for (int off = 16; off >= 1; off >>= 1)
            for (int l = 0; l < off; ++l) reference_node(rs[l], rc[l], rs[l + off], rc[l + off]);
        const double ref_c = hk::ss::finite(rs[0]) ? rc[0] : 0.0;

        double ds[32], dc[32];
        for (int l = 0; l < 32; ++l) ds[l] = x[l], dc[l] = 0.0;
        for (int l = 0; l < 16; ++l) {
            const bool swap = next() & 1;
            const double a = swap ? ds[l + 16] : ds[l], b = swap ? ds[l] : ds[l + 16];
            const double t = a + b;
            dc[l] = hk::ss::two_sum_err(a, b, t);
            ds[l] = t;
        }
        for (int off = 8; off >= 1; off >>= 1)
            for (int l = 0; l < off; ++l) {
                if (next() & 1) {
                    hk::ss::pair_combine_unchecked<hk::ss::kSum>(ds[l], dc[l], ds[l + off], dc[l + off]);
                } else {
                    double s = ds[l + off], c = dc[l + off];
                    hk::ss::pair_combine_unchecked<hk::ss::kSum>(s, c, ds[l], dc[l]);
                    ds[l] = s, dc[l] = c;
                }
            }
        const double dev_c = hk::ss::root_comp<hk::ss::kSum>(ds[0], dc[0]);
        if (!same(rs[0], ds[0]) || !same(ref_c, dev_c)) {
            if (bad < 5)
                std::printf("row %ld: reference (%a, %a) device (%a, %a)\n", r, rs[0], ref_c, ds[0], dev_c);
            ++bad;
        }
    }
    std::printf("mismatches %ld of %ld rows\n", bad, rows);
    return bad == 0 ? 0 : 1;
}
