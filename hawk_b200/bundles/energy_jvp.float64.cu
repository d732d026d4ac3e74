// hawk_b200 unit 'energy_jvp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(128, 13) energy_jvp(
    hk::abi::ScalarHandle p_mut_dot_out,
    hk::abi::GRefMirror p_vin_dot_v,
    hk::abi::GRefMirror p_vin_v,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_dot_out(p_mut_dot_out);
    (void)mut_dot_out;
    const hk::VecIn<Real, 3> vin_dot_v(p_vin_dot_v);
    (void)vin_dot_v;
    const hk::VecIn<Real, 3> vin_v(p_vin_v);
    (void)vin_v;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto vin_dot_v_i = vin_dot_v[i].get();
        const auto vin_v_i = vin_v[i].get();
        mut_dot_out[i] = (static_cast<Real>(0.5) * (vin_dot_v_i.dot(vin_v_i) + vin_v_i.dot(vin_dot_v_i)));
    }
}
