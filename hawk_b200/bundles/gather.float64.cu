// hawk_b200 unit 'gather' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) gather(
    hk::abi::ScalarHandle p_mut_y,
    hk::abi::ScalarHandle p_psc_idx,
    hk::abi::ScalarHandle p_psc_w,
    hk::abi::ScalarHandle p_lut_table,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_y(p_mut_y);
    (void)mut_y;
    const hk::ScalarIn<std::int32_t> psc_idx(p_psc_idx);
    (void)psc_idx;
    const hk::ScalarIn<Real> psc_w(p_psc_w);
    (void)psc_w;
    const hk::ScalarIn<Real> lut_table(p_lut_table);
    (void)lut_table;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        mut_y[i] = (psc_w[i].eval() * lut_table[hk::SampleIndex::make(static_cast<std::size_t>(hawk_abi::int_clamp_index<Int>(static_cast<Int>(psc_idx[i].eval()), static_cast<Int>(lut_table.samples()))))].eval());
    }
}
