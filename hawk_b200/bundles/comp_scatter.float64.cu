// hawk_b200 unit 'comp_scatter' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__comp_scatter = 32768u;
extern "C" __global__ void __launch_bounds__(256) comp_scatter(
    hk::abi::ScalarHandle p_aout_acc,
    hk::abi::ScalarHandle p_aout_acc_c,
    hk::abi::ScalarHandle p_psc_key,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_acc(p_aout_acc);
    (void)aout_acc;
    const hk::ScalarOut<Real> aout_acc_c(p_aout_acc_c);
    (void)aout_acc_c;
    const hk::ScalarIn<std::int32_t> psc_key(p_psc_key);
    (void)psc_key;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    hk::accum::PrivSpace hawk_ps = hk::accum::private_space();
    const auto hawk_pv_aout_acc = hk::accum::privatise(hawk_ps, aout_acc);
    const auto hawk_pv_aout_acc_c = hk::accum::privatise(hawk_ps, aout_acc_c);
    __syncthreads();
    {
    const auto& aout_acc = hawk_pv_aout_acc;
    const auto& aout_acc_c = hawk_pv_aout_acc_c;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto t2 = static_cast<Int>(psc_key[i].eval());
        hawk_abi::accum_add_compensated(aout_acc, aout_acc_c, hk::SampleIndex::make(static_cast<std::size_t>(t2)), psc_x[i].eval());
    }
    }
    __syncthreads();
    hk::accum::flush_compensated(hawk_pv_aout_acc, hawk_pv_aout_acc_c);
}
