// hawk_b200 unit 'gravity' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(128, 11) gravity(
    hk::abi::GRefMirror p_mut_f,
    hk::abi::ScalarHandle p_mut_u,
    hk::abi::GRefMirror p_vin_r1,
    hk::abi::GRefMirror p_vin_r2,
    hk::abi::ScalarHandle p_psc_m1,
    hk::abi::ScalarHandle p_psc_m2,
    Real p_uni_G,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::VecOut<Real, 3> mut_f(p_mut_f);
    (void)mut_f;
    const hk::ScalarOut<Real> mut_u(p_mut_u);
    (void)mut_u;
    const hk::VecIn<Real, 3> vin_r1(p_vin_r1);
    (void)vin_r1;
    const hk::VecIn<Real, 3> vin_r2(p_vin_r2);
    (void)vin_r2;
    const hk::ScalarIn<Real> psc_m1(p_psc_m1);
    (void)psc_m1;
    const hk::ScalarIn<Real> psc_m2(p_psc_m2);
    (void)psc_m2;
    const Real uni_G = p_uni_G;
    (void)uni_G;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto t4 = ((uni_G * psc_m1[i].eval()) * psc_m2[i].eval());
        const auto vin_r2_i = vin_r2[i].get();
        const auto vin_r1_i = vin_r1[i].get();
        const hk::Item<Real, 3> t7 = (vin_r2_i - vin_r1_i);
        const auto t8 = t7.norm();
        mut_f[i] = (static_cast<Real>((t4 / ((t8 * t8) * t8))) * t7);
        mut_u[i] = ((-t4) / t8);
    }
}
