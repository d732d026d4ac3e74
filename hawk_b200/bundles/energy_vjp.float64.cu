// hawk_b200 unit 'energy_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) energy_vjp(
    hk::abi::GRefMirror p_mut_bar_v,
    hk::abi::GRefMirror p_vin_v,
    hk::abi::ScalarHandle p_psc_bar_out,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::VecOut<Real, 3> mut_bar_v(p_mut_bar_v);
    (void)mut_bar_v;
    const hk::VecIn<Real, 3> vin_v(p_vin_v);
    (void)vin_v;
    const hk::ScalarIn<Real> psc_bar_out(p_psc_bar_out);
    (void)psc_bar_out;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto vin_v_i = vin_v[i].get();
        const hk::Item<Real, 3> t4 = (static_cast<Real>((psc_bar_out[i].eval() * static_cast<Real>(0.5))) * vin_v_i);
        mut_bar_v[i] = (t4 + t4);
    }
}
