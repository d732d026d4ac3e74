// hawk_b200 unit 'key_total' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) key_total(
    hk::abi::ScalarHandle p_aout_out,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_out(p_aout_out);
    (void)aout_out;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    hk::accum::run::State hawk_run_aout_out{};
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        hk::accum::run::add<8>(aout_out, hk::SampleIndex::make(static_cast<std::size_t>((static_cast<Int>(hawk_i) / static_cast<Int>(8)))), psc_x[i].eval(), i, hawk_run_aout_out);
    }
}
