// hawk_b200 unit 'poly_loss' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) poly_loss(
    hk::abi::ScalarHandle p_mut_r,
    hk::abi::ScalarHandle p_psc_t,
    hk::abi::ScalarHandle p_psc_x,
    Real p_uni_a,
    Real p_uni_b,
    Real p_uni_c,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_r(p_mut_r);
    (void)mut_r;
    const hk::ScalarIn<Real> psc_t(p_psc_t);
    (void)psc_t;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const Real uni_a = p_uni_a;
    (void)uni_a;
    const Real uni_b = p_uni_b;
    (void)uni_b;
    const Real uni_c = p_uni_c;
    (void)uni_c;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto t11 = ((((((uni_a * psc_x_i) * psc_x_i) * psc_x_i) + (uni_b * psc_x_i)) + uni_c) - psc_t[i].eval());
        mut_r[i] = (t11 * t11);
    }
}
