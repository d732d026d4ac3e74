// hawk_b200 unit 'gravity_jvp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) gravity_jvp(
    hk::abi::GRefMirror p_mut_dot_f,
    hk::abi::ScalarHandle p_mut_dot_u,
    hk::abi::GRefMirror p_vin_dot_r1,
    hk::abi::GRefMirror p_vin_dot_r2,
    hk::abi::GRefMirror p_vin_r1,
    hk::abi::GRefMirror p_vin_r2,
    hk::abi::ScalarHandle p_psc_m1,
    hk::abi::ScalarHandle p_psc_m2,
    Real p_uni_G,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::VecOut<Real, 3> mut_dot_f(p_mut_dot_f);
    (void)mut_dot_f;
    const hk::ScalarOut<Real> mut_dot_u(p_mut_dot_u);
    (void)mut_dot_u;
    const hk::VecIn<Real, 3> vin_dot_r1(p_vin_dot_r1);
    (void)vin_dot_r1;
    const hk::VecIn<Real, 3> vin_dot_r2(p_vin_dot_r2);
    (void)vin_dot_r2;
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
        const auto t9 = (t8 * t8);
        const auto t10 = (t9 * t8);
        const auto t11 = (t4 / t10);
        const auto vin_dot_r2_i = vin_dot_r2[i].get();
        const auto vin_dot_r1_i = vin_dot_r1[i].get();
        const hk::Item<Real, 3> t15 = (vin_dot_r2_i + (vin_dot_r1_i * static_cast<Real>(-1)));
        const auto t17 = (t7.dot(t15) / t8);
        mut_dot_f[i] = ((static_cast<Real>((-((t11 * ((((t17 * t8) + (t8 * t17)) * t8) + (t9 * t17))) / t10))) * t7) + (static_cast<Real>(t11) * t15));
        mut_dot_u[i] = (-((((-t4) / t8) * t17) / t8));
    }
}
