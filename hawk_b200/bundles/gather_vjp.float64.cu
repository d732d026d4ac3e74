// hawk_b200 unit 'gather_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__gather_vjp = 32768u;
extern "C" __global__ void __launch_bounds__(256) gather_vjp(
    hk::abi::ScalarHandle p_mut_bar_w,
    hk::abi::ScalarHandle p_aout_bar_table,
    hk::abi::ScalarHandle p_psc_bar_y,
    hk::abi::ScalarHandle p_psc_idx,
    hk::abi::ScalarHandle p_psc_w,
    hk::abi::ScalarHandle p_lut_table,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_bar_w(p_mut_bar_w);
    (void)mut_bar_w;
    const hk::ScalarOut<Real> aout_bar_table(p_aout_bar_table);
    (void)aout_bar_table;
    const hk::ScalarIn<Real> psc_bar_y(p_psc_bar_y);
    (void)psc_bar_y;
    const hk::ScalarIn<std::int32_t> psc_idx(p_psc_idx);
    (void)psc_idx;
    const hk::ScalarIn<Real> psc_w(p_psc_w);
    (void)psc_w;
    const hk::ScalarIn<Real> lut_table(p_lut_table);
    (void)lut_table;
    hk::accum::PrivSpace hawk_ps = hk::accum::private_space();
    const auto hawk_pv_aout_bar_table = hk::accum::privatise(hawk_ps, aout_bar_table);
    __syncthreads();
    {
    const auto& aout_bar_table = hawk_pv_aout_bar_table;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_bar_y_i = psc_bar_y[i].eval();
        const auto t5 = hawk_abi::int_clamp_index<Int>(static_cast<Int>(psc_idx[i].eval()), static_cast<Int>(lut_table.samples()));
        mut_bar_w[i] = (psc_bar_y_i * lut_table[hk::SampleIndex::make(static_cast<std::size_t>(t5))].eval());
        hawk_abi::accum_add(aout_bar_table, hk::SampleIndex::make(static_cast<std::size_t>(t5)), (psc_bar_y_i * psc_w[i].eval()));
    }
    }
    __syncthreads();
    hk::accum::flush_add(hawk_pv_aout_bar_table);
}
