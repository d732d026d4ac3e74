// hawk_b200 unit 'band_chain' (scalar mode banded), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) band_chain(
    hk::abi::ScalarHandle p_mut_out,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_psc_y,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_out(p_mut_out);
    (void)mut_out;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> psc_y(p_psc_y);
    (void)psc_y;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto psc_y_i = psc_y[i].eval();
        mut_out[i] = ((hk::math::exp((((psc_x_i * psc_x_i) * static_cast<Real>(0.5)) + psc_y_i)) / (psc_y_i + static_cast<Real>(1.5))) - (hk::math::sin(psc_x_i) * static_cast<Real>(0.25)));
    }
}
