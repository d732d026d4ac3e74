// hawk_b200 unit 'trig' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) trig(
    hk::abi::ScalarHandle p_mut_c,
    hk::abi::ScalarHandle p_mut_s,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_c(p_mut_c);
    (void)mut_c;
    const hk::ScalarOut<Real> mut_s(p_mut_s);
    (void)mut_s;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        mut_s[i] = hk::math::sin(psc_x_i);
        mut_c[i] = hk::math::cos(psc_x_i);
    }
}
