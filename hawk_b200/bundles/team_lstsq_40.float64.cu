// hawk_b200 unit 'team_lstsq_40' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_team_threads__team_lstsq_40 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_lstsq_40 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_lstsq_40(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_r0,
    hk::abi::GRefMirror p_vin_r,
    hk::abi::GRefMirror p_mtx_J,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<Real> wout_tm0_r0(p_wout_tm0_r0);
    (void)wout_tm0_r0;
    const hk::VecIn<Real, 80> vin_r(p_vin_r);
    (void)vin_r;
    const hk::MatIn<Real, 80, 40> mtx_J(p_mtx_J);
    (void)mtx_J;
    hk::linalg::team::begin_entry();
    const long long hawk_teams = static_cast<long long>(blockDim.x >> 5);
    for (long long hawk_flat = static_cast<long long>(blockIdx.x) * hawk_teams + (threadIdx.x >> 5); hawk_flat < count; hawk_flat += static_cast<long long>(gridDim.x) * hawk_teams) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        const Int hawk_wl = static_cast<Int>(threadIdx.x & 31);
        (void)hawk_i;
        (void)hawk_wl;
        (void)nSamples;
        const auto mtx_J_i = mtx_J[i].get();
        const auto vin_r_i = vin_r[i].get();
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 3200; hawk_lk += hawk_tm.size) wout_tm0_a.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 3200 + hawk_lk] = mtx_J[i].at(hawk_lk / 40, hawk_lk % 40); }
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 80; hawk_lk += hawk_tm.size) wout_tm0_r0.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 80 + hawk_lk] = vin_r[i].at(hawk_lk); }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_lstsq_40_2 = 32u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_lstsq_40_2 = 13888u;
extern "C" __global__ void __launch_bounds__(32) team_lstsq_40_2(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_info,
    hk::abi::ScalarHandle p_wout_tm0_r0,
    hk::abi::ScalarHandle p_wout_tm0_tau,
    hk::abi::ScalarHandle p_wout_tm0_work,
    hk::abi::ScalarHandle p_wout_tm0_x0,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<std::int32_t> wout_tm0_info(p_wout_tm0_info);
    (void)wout_tm0_info;
    const hk::ScalarOut<Real> wout_tm0_r0(p_wout_tm0_r0);
    (void)wout_tm0_r0;
    const hk::ScalarOut<Real> wout_tm0_tau(p_wout_tm0_tau);
    (void)wout_tm0_tau;
    const hk::ScalarOut<Real> wout_tm0_work(p_wout_tm0_work);
    (void)wout_tm0_work;
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
        {  // qr, n = 40
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 3200;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            Real* const hawk_tau = wout_tm0_tau.data() + static_cast<std::size_t>(hawk_lane) * 40;
            Real* const hawk_work = wout_tm0_work.data() + static_cast<std::size_t>(hawk_lane) * 81;
            const auto hawk_f = hk::linalg::team::TeamQr<Real, 40>{hawk_a, hawk_tau, hawk_work, hawk_info};
            hk::linalg::team::qr<40>(hawk_tm, hawk_f, hawk_a, 80);
        }
        {  // qr_solve, n = 40
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 3200;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            Real* const hawk_tau = wout_tm0_tau.data() + static_cast<std::size_t>(hawk_lane) * 40;
            Real* const hawk_work = wout_tm0_work.data() + static_cast<std::size_t>(hawk_lane) * 81;
            Real* const hawk_r = wout_tm0_r0.data() + static_cast<std::size_t>(hawk_lane) * 80;
            Real* const hawk_x = wout_tm0_x0.data() + static_cast<std::size_t>(hawk_lane) * 40;
            const auto hawk_f = hk::linalg::team::TeamQr<Real, 40>{hawk_a, hawk_tau, hawk_work, hawk_info};
            hk::linalg::team::qrSolve<40>(hawk_tm, hawk_f, 80, hawk_r, hawk_x, 1);
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_lstsq_40_3 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_lstsq_40_3 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_lstsq_40_3(
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
    const hk::VecOut<Real, 40> mut_x(p_mut_x);
    (void)mut_x;
    const hk::ScalarIn<std::int32_t> lut_tm0_info(p_lut_tm0_info);
    (void)lut_tm0_info;
    const hk::ScalarIn<Real> lut_tm0_x0(p_lut_tm0_x0);
    (void)lut_tm0_x0;
    __shared__ __align__(16) unsigned char hk_tile[32 * 33 * 8];
    const long long hk_lane_tiles = (count + 31) / 32;
    const long long hk_end0 = hk_lane_tiles * 2;
    const long long hk_end1 = hk_end0 + hk_lane_tiles * 1;
    for (long long hk_t = blockIdx.x; hk_t < hk_end1; hk_t += gridDim.x) {
        if (hk_t < hk_end0) hk::linalg::team::copyOutTile(lut_tm0_x0.data(), mut_x.data(), mut_x.pitch, 40LL, base, count, hk_t, hk_tile);
        else hk::linalg::team::copyOutTile(lut_tm0_info.data(), mut_info.data(), 0ull, 1LL, base, count, hk_t - hk_end0, hk_tile);
    }
    (void)nSamples;
}
