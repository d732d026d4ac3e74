// hawk_b200 unit 'team_chol_512' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#define HK_TEAM_LOWER_STAGED 0
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_team_threads__team_chol_512 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_chol_512 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_chol_512(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_x0,
    hk::abi::GRefMirror p_vin_b,
    hk::abi::GRefMirror p_mtx_A,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<Real> wout_tm0_x0(p_wout_tm0_x0);
    (void)wout_tm0_x0;
    const hk::VecIn<Real, 512> vin_b(p_vin_b);
    (void)vin_b;
    const hk::MatIn<Real, 512, 512> mtx_A(p_mtx_A);
    (void)mtx_A;
    hk::linalg::team::begin_entry();
    const long long hawk_teams = static_cast<long long>(blockDim.x >> 5);
    for (long long hawk_flat = static_cast<long long>(blockIdx.x) * hawk_teams + (threadIdx.x >> 5); hawk_flat < count; hawk_flat += static_cast<long long>(gridDim.x) * hawk_teams) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        const Int hawk_wl = static_cast<Int>(threadIdx.x & 31);
        (void)hawk_i;
        (void)hawk_wl;
        (void)nSamples;
        const auto mtx_A_i = mtx_A[i].get();
        const auto vin_b_i = vin_b[i].get();
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 262144; hawk_lk += hawk_tm.size) wout_tm0_a.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 262144 + hawk_lk] = mtx_A[i].at(hawk_lk / 512, hawk_lk % 512); }
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 512; hawk_lk += hawk_tm.size) wout_tm0_x0.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 512 + hawk_lk] = vin_b[i].at(hawk_lk); }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_chol_512_2 = 128u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_chol_512_2 = 16896u;
extern "C" __global__ void __launch_bounds__(128) team_chol_512_2(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_info,
    hk::abi::ScalarHandle p_wout_tm0_x0,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<std::int32_t> wout_tm0_info(p_wout_tm0_info);
    (void)wout_tm0_info;
    const hk::ScalarOut<Real> wout_tm0_x0(p_wout_tm0_x0);
    (void)wout_tm0_x0;
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
        {  // chol, n = 512
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 262144;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            const auto hawk_f = hk::linalg::team::TeamCholesky<Real, 512>{hawk_a, hawk_info};
            hk::linalg::team::cholesky<512>(hawk_tm, hawk_f, hawk_a);
        }
        {  // cho_solve, n = 512
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 262144;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            Real* const hawk_x = wout_tm0_x0.data() + static_cast<std::size_t>(hawk_lane) * 512;
            const auto hawk_f = hk::linalg::team::TeamCholesky<Real, 512>{hawk_a, hawk_info};
            hk::linalg::team::choSolve<512>(hawk_tm, hawk_f, hawk_x, hawk_x, 1);
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_chol_512_3 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_chol_512_3 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_chol_512_3(
    hk::abi::ScalarHandle p_mut_info,
    hk::abi::GRefMirror p_mut_x,
    hk::abi::ScalarHandle p_lut_tm0_info,
    hk::abi::ScalarHandle p_lut_tm0_x0,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<std::int32_t> mut_info(p_mut_info);
    (void)mut_info;
    const hk::VecOut<Real, 512> mut_x(p_mut_x);
    (void)mut_x;
    const hk::ScalarIn<std::int32_t> lut_tm0_info(p_lut_tm0_info);
    (void)lut_tm0_info;
    const hk::ScalarIn<Real> lut_tm0_x0(p_lut_tm0_x0);
    (void)lut_tm0_x0;
    __shared__ __align__(16) unsigned char hk_tile[32 * 33 * 8];
    const long long hk_lane_tiles = (count + 31) / 32;
    const long long hk_end0 = hk_lane_tiles * 16;
    const long long hk_end1 = hk_end0 + hk_lane_tiles * 1;
    for (long long hk_t = blockIdx.x; hk_t < hk_end1; hk_t += gridDim.x) {
        if (hk_t < hk_end0) hk::linalg::team::copyOutTile(lut_tm0_x0.data(), mut_x.data(), mut_x.pitch, 512LL, base, count, hk_t, hk_tile);
        else hk::linalg::team::copyOutTile(lut_tm0_info.data(), mut_info.data(), 0ull, 1LL, base, count, hk_t - hk_end0, hk_tile);
    }
    (void)nSamples;
}
