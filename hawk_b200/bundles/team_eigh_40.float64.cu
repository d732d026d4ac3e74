// hawk_b200 unit 'team_eigh_40' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_team_threads__team_eigh_40 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_eigh_40 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_eigh_40(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::GRefMirror p_mtx_A,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::MatIn<Real, 40, 40> mtx_A(p_mtx_A);
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
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 1600; hawk_lk += hawk_tm.size) wout_tm0_a.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 1600 + hawk_lk] = mtx_A[i].at(hawk_lk / 40, hawk_lk % 40); }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_eigh_40_2 = 32u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_eigh_40_2 = 13888u;
extern "C" __global__ void __launch_bounds__(32) team_eigh_40_2(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_info,
    hk::abi::ScalarHandle p_wout_tm0_v,
    hk::abi::ScalarHandle p_wout_tm0_w,
    hk::abi::ScalarHandle p_wout_tm0_work,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<std::int32_t> wout_tm0_info(p_wout_tm0_info);
    (void)wout_tm0_info;
    const hk::ScalarOut<Real> wout_tm0_v(p_wout_tm0_v);
    (void)wout_tm0_v;
    const hk::ScalarOut<Real> wout_tm0_w(p_wout_tm0_w);
    (void)wout_tm0_w;
    const hk::ScalarOut<Real> wout_tm0_work(p_wout_tm0_work);
    (void)wout_tm0_work;
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
        {  // eigh, n = 40
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 1600;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            Real* const hawk_w = wout_tm0_w.data() + static_cast<std::size_t>(hawk_lane) * 40;
            Real* const hawk_v = wout_tm0_v.data() + static_cast<std::size_t>(hawk_lane) * 1600;
            Real* const hawk_work = wout_tm0_work.data() + static_cast<std::size_t>(hawk_lane) * 1604;
            const auto hawk_f = hk::linalg::team::TeamEigh<Real, 40>{hawk_w, hawk_v, hawk_work, hawk_info};
            hk::linalg::team::eigh<40>(hawk_tm, hawk_f, hawk_a);
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_eigh_40_3 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_eigh_40_3 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_eigh_40_3(
    hk::abi::GRefMirror p_mut_V,
    hk::abi::ScalarHandle p_mut_info,
    hk::abi::GRefMirror p_mut_w,
    hk::abi::ScalarHandle p_lut_tm0_info,
    hk::abi::ScalarHandle p_lut_tm0_v,
    hk::abi::ScalarHandle p_lut_tm0_w,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::MatOut<Real, 40, 40> mut_V(p_mut_V);
    (void)mut_V;
    const hk::ScalarOut<std::int32_t> mut_info(p_mut_info);
    (void)mut_info;
    const hk::VecOut<Real, 40> mut_w(p_mut_w);
    (void)mut_w;
    const hk::ScalarIn<std::int32_t> lut_tm0_info(p_lut_tm0_info);
    (void)lut_tm0_info;
    const hk::ScalarIn<Real> lut_tm0_v(p_lut_tm0_v);
    (void)lut_tm0_v;
    const hk::ScalarIn<Real> lut_tm0_w(p_lut_tm0_w);
    (void)lut_tm0_w;
    __shared__ __align__(16) unsigned char hk_tile[32 * 33 * 8];
    const long long hk_lane_tiles = (count + 31) / 32;
    const long long hk_end0 = hk_lane_tiles * 2;
    const long long hk_end1 = hk_end0 + hk_lane_tiles * 50;
    const long long hk_end2 = hk_end1 + hk_lane_tiles * 1;
    for (long long hk_t = blockIdx.x; hk_t < hk_end2; hk_t += gridDim.x) {
        if (hk_t < hk_end0) hk::linalg::team::copyOutTile(lut_tm0_w.data(), mut_w.data(), mut_w.pitch, 40LL, base, count, hk_t, hk_tile);
        else if (hk_t < hk_end1) hk::linalg::team::copyOutTile(lut_tm0_v.data(), mut_V.data(), mut_V.pitch, 1600LL, base, count, hk_t - hk_end0, hk_tile);
        else hk::linalg::team::copyOutTile(lut_tm0_info.data(), mut_info.data(), 0ull, 1LL, base, count, hk_t - hk_end1, hk_tile);
    }
    (void)nSamples;
}
