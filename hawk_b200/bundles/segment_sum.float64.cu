// hawk_b200 unit 'segment_sum' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) segment_sum(
    hk::abi::ScalarHandle p_aout_acc,
    hk::abi::ScalarHandle p_aout_acc_c,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_acc(p_aout_acc);
    (void)aout_acc;
    const hk::ScalarOut<Real> aout_acc_c(p_aout_acc_c);
    (void)aout_acc_c;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    hk::accum::run::State hawk_run_aout_acc{};
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto t3 = (static_cast<Int>(hawk_i) / static_cast<Int>(256));
        hk::accum::run::addCompensated<32>(aout_acc, aout_acc_c, hk::SampleIndex::make(static_cast<std::size_t>(t3)), psc_x[i].eval(), i, hawk_run_aout_acc);
    }
}

extern "C" __global__ void __launch_bounds__(256) segment_sum__fold_acc(
    hk::abi::ScalarHandle p_aout_acc,
    hk::abi::ScalarHandle p_aout_acc_c,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_acc(p_aout_acc);
    (void)aout_acc;
    const hk::ScalarOut<Real> aout_acc_c(p_aout_acc_c);
    (void)aout_acc_c;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        hawk_abi::fold_companion(aout_acc, aout_acc_c, i);
    }
}
