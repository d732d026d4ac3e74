// hawk_b200 unit 'gravity_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) gravity_vjp(
    hk::abi::GRefMirror p_mut_bar_r1,
    hk::abi::GRefMirror p_mut_bar_r2,
    hk::abi::GRefMirror p_vin_bar_f,
    hk::abi::GRefMirror p_vin_r1,
    hk::abi::GRefMirror p_vin_r2,
    hk::abi::ScalarHandle p_psc_bar_u,
    hk::abi::ScalarHandle p_psc_m1,
    hk::abi::ScalarHandle p_psc_m2,
    Real p_uni_G,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::VecOut<Real, 3> mut_bar_r1(p_mut_bar_r1);
    (void)mut_bar_r1;
    const hk::VecOut<Real, 3> mut_bar_r2(p_mut_bar_r2);
    (void)mut_bar_r2;
    const hk::VecIn<Real, 3> vin_bar_f(p_vin_bar_f);
    (void)vin_bar_f;
    const hk::VecIn<Real, 3> vin_r1(p_vin_r1);
    (void)vin_r1;
    const hk::VecIn<Real, 3> vin_r2(p_vin_r2);
    (void)vin_r2;
    const hk::ScalarIn<Real> psc_bar_u(p_psc_bar_u);
    (void)psc_bar_u;
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
        const auto vin_bar_f_i = vin_bar_f[i].get();
        const auto t5 = ((uni_G * psc_m1[i].eval()) * psc_m2[i].eval());
        const auto vin_r2_i = vin_r2[i].get();
        const auto vin_r1_i = vin_r1[i].get();
        const hk::Item<Real, 3> t8 = (vin_r2_i - vin_r1_i);
        const auto t9 = t8.norm();
        const auto t10 = (t9 * t9);
        const auto t11 = (t10 * t9);
        const auto t12 = (t5 / t11);
        const auto t24 = (-((vin_bar_f_i.cwiseMul(t8).sum() * t12) / t11));
        const auto t28 = ((t24 * t9) * t9);
        const hk::Item<Real, 3> t33 = ((vin_bar_f_i * static_cast<Real>(t12)) + (static_cast<Real>((((((-((psc_bar_u[i].eval() * ((-t5) / t9)) / t9)) + (t24 * t10)) + t28) + t28) / t9)) * t8));
        mut_bar_r2[i] = t33;
        mut_bar_r1[i] = (t33 * static_cast<Real>(-1));
    }
}
