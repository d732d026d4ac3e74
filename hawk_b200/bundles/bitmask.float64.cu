// hawk_b200 unit 'bitmask' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__bitmask = 32768u;
extern "C" __global__ void __launch_bounds__(256) bitmask(
    hk::abi::ScalarHandle p_aout_acc,
    hk::abi::ScalarHandle p_psc_bits,
    hk::abi::ScalarHandle p_psc_key,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<std::uint32_t> aout_acc(p_aout_acc);
    (void)aout_acc;
    const hk::ScalarIn<std::uint32_t> psc_bits(p_psc_bits);
    (void)psc_bits;
    const hk::ScalarIn<std::int32_t> psc_key(p_psc_key);
    (void)psc_key;
    hk::accum::PrivSpace hawk_ps = hk::accum::private_space();
    const auto hawk_pv_aout_acc = hk::accum::privatise(hawk_ps, aout_acc);
    __syncthreads();
    {
    const auto& aout_acc = hawk_pv_aout_acc;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        hawk_abi::accum_or(aout_acc, hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(psc_key[i].eval()))), psc_bits[i].eval());
    }
    }
    __syncthreads();
    hk::accum::flush_or(hawk_pv_aout_acc);
}
