// hawk_b200 unit 'key_share' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) key_share(
    hk::abi::ScalarHandle p_aout_cut0,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_cut0(p_aout_cut0);
    (void)aout_cut0;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    hk::accum::run::State hawk_run_aout_cut0{};
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        hk::accum::run::add<8>(aout_cut0, hk::SampleIndex::make(static_cast<std::size_t>((static_cast<Int>(hawk_i) / static_cast<Int>(8)))), psc_x[i].eval(), i, hawk_run_aout_cut0);
    }
}

extern "C" __global__ void __launch_bounds__(256) key_share_2(
    hk::abi::ScalarHandle p_mut_z,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_lut_cut0,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_z(p_mut_z);
    (void)mut_z;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> lut_cut0(p_lut_cut0);
    (void)lut_cut0;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        mut_z[i] = (psc_x[i].eval() / lut_cut0[hk::SampleIndex::make(static_cast<std::size_t>((static_cast<Int>(hawk_i) / static_cast<Int>(8))))].eval());
    }
}
