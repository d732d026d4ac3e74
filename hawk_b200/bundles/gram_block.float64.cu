// hawk_b200 unit 'gram_block' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) gram_block(
    hk::abi::ScalarHandle p_wout_tmb0_u,
    hk::abi::GRefMirror p_vin_j,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tmb0_u(p_wout_tmb0_u);
    (void)wout_tmb0_u;
    const hk::VecIn<Real, 6> vin_j(p_vin_j);
    (void)vin_j;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto vin_j_i = vin_j[i].get();
        for (Int hawk_lk = 0; hawk_lk < 6; ++hawk_lk) wout_tmb0_u.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 6 + hawk_lk] = vin_j[i].at(hawk_lk);
    }
}

extern "C" __device__ const unsigned int hk_team_threads__gram_block_2 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__gram_block_2 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__gram_block_2 = 800u;
extern "C" __global__ void __launch_bounds__(32) gram_block_2(
    hk::abi::ScalarHandle p_wout_out,
    hk::abi::ScalarHandle p_wout_tmb0_u,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_out(p_wout_out);
    (void)wout_out;
    const hk::ScalarOut<Real> wout_tmb0_u(p_wout_tmb0_u);
    (void)wout_tmb0_u;
    hk::linalg::team::begin_entry();
    const long long hawk_teams = static_cast<long long>(blockDim.x >> 5);
    for (long long hawk_flat = static_cast<long long>(blockIdx.x) * hawk_teams + (threadIdx.x >> 5); hawk_flat < count; hawk_flat += static_cast<long long>(gridDim.x) * hawk_teams) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        const Int hawk_wl = static_cast<Int>(threadIdx.x & 31);
        (void)hawk_i;
        (void)hawk_wl;
        (void)nSamples;
        const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here();
        const long long hawk_lane = hawk_i;
        {  // block_sum, n = 6
            const std::size_t hawk_key = static_cast<std::size_t>(hawk_lane);
            const std::size_t hawk_keys = static_cast<std::size_t>(count);
            const std::size_t hawk_rows = static_cast<std::size_t>(nSamples) / hawk_keys;
            const Real* const hawk_u = wout_tmb0_u.data();
            const Real* const hawk_v = wout_tmb0_u.data();
            Real* const hawk_out = wout_out.data();
            hk::linalg::team::blockSum<6, 6>(hawk_tm, hawk_out + hawk_key, hawk_u, hawk_v, hawk_key * hawk_rows, hawk_rows, 6, 6, nullptr, 6 * hawk_keys, hawk_keys, 1);
        }
        __syncwarp();
    }
}
