// hawk_b200 unit 'team_lu_33' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_team_threads__team_lu_33 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_lu_33 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_lu_33(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_x0,
    hk::abi::ScalarHandle p_wout_tm0_x1,
    hk::abi::ScalarHandle p_wout_tm1_a,
    hk::abi::GRefMirror p_vin_b,
    hk::abi::GRefMirror p_mtx_A,
    hk::abi::GRefMirror p_mtx_B,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<Real> wout_tm0_x0(p_wout_tm0_x0);
    (void)wout_tm0_x0;
    const hk::ScalarOut<Real> wout_tm0_x1(p_wout_tm0_x1);
    (void)wout_tm0_x1;
    const hk::ScalarOut<Real> wout_tm1_a(p_wout_tm1_a);
    (void)wout_tm1_a;
    const hk::VecIn<Real, 33> vin_b(p_vin_b);
    (void)vin_b;
    const hk::MatIn<Real, 33, 33> mtx_A(p_mtx_A);
    (void)mtx_A;
    const hk::MatIn<Real, 33, 2> mtx_B(p_mtx_B);
    (void)mtx_B;
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
        const auto mtx_B_i = mtx_B[i].get();
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 1089; hawk_lk += hawk_tm.size) wout_tm0_a.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 1089 + hawk_lk] = mtx_A[i].at(hawk_lk / 33, hawk_lk % 33); }
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 33; hawk_lk += hawk_tm.size) wout_tm0_x0.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 33 + hawk_lk] = vin_b[i].at(hawk_lk); }
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 66; hawk_lk += hawk_tm.size) wout_tm0_x1.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 66 + hawk_lk] = mtx_B[i].at(hawk_lk / 2, hawk_lk % 2); }
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 1089; hawk_lk += hawk_tm.size) wout_tm1_a.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 1089 + hawk_lk] = mtx_A[i].at(hawk_lk / 33, hawk_lk % 33); }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_lu_33_2 = 32u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_lu_33_2 = 9904u;
extern "C" __global__ void __launch_bounds__(32) team_lu_33_2(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_info,
    hk::abi::ScalarHandle p_wout_tm0_piv,
    hk::abi::ScalarHandle p_wout_tm0_x0,
    hk::abi::ScalarHandle p_wout_tm0_x1,
    hk::abi::ScalarHandle p_wout_tm1_a,
    hk::abi::ScalarHandle p_wout_tm1_d0,
    hk::abi::ScalarHandle p_wout_tm1_info,
    hk::abi::ScalarHandle p_wout_tm1_piv,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<std::int32_t> wout_tm0_info(p_wout_tm0_info);
    (void)wout_tm0_info;
    const hk::ScalarOut<std::int32_t> wout_tm0_piv(p_wout_tm0_piv);
    (void)wout_tm0_piv;
    const hk::ScalarOut<Real> wout_tm0_x0(p_wout_tm0_x0);
    (void)wout_tm0_x0;
    const hk::ScalarOut<Real> wout_tm0_x1(p_wout_tm0_x1);
    (void)wout_tm0_x1;
    const hk::ScalarOut<Real> wout_tm1_a(p_wout_tm1_a);
    (void)wout_tm1_a;
    const hk::ScalarOut<Real> wout_tm1_d0(p_wout_tm1_d0);
    (void)wout_tm1_d0;
    const hk::ScalarOut<std::int32_t> wout_tm1_info(p_wout_tm1_info);
    (void)wout_tm1_info;
    const hk::ScalarOut<std::int32_t> wout_tm1_piv(p_wout_tm1_piv);
    (void)wout_tm1_piv;
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
        {  // lu, n = 33
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 1089;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            std::int32_t* const hawk_piv = wout_tm0_piv.data() + static_cast<std::size_t>(hawk_lane) * 33;
            const auto hawk_f = hk::linalg::team::TeamLu<Real, 33>{hawk_a, hawk_piv, hawk_info};
            hk::linalg::team::lu<33>(hawk_tm, hawk_f, hawk_a);
        }
        {  // lu_solve, n = 33
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 1089;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            std::int32_t* const hawk_piv = wout_tm0_piv.data() + static_cast<std::size_t>(hawk_lane) * 33;
            Real* const hawk_x = wout_tm0_x0.data() + static_cast<std::size_t>(hawk_lane) * 33;
            const auto hawk_f = hk::linalg::team::TeamLu<Real, 33>{hawk_a, hawk_piv, hawk_info};
            hk::linalg::team::luSolve<33>(hawk_tm, hawk_f, hawk_x, hawk_x, 1);
        }
        {  // lu_solve, n = 33
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 1089;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            std::int32_t* const hawk_piv = wout_tm0_piv.data() + static_cast<std::size_t>(hawk_lane) * 33;
            Real* const hawk_x = wout_tm0_x1.data() + static_cast<std::size_t>(hawk_lane) * 66;
            const auto hawk_f = hk::linalg::team::TeamLu<Real, 33>{hawk_a, hawk_piv, hawk_info};
            hk::linalg::team::luSolve<33>(hawk_tm, hawk_f, hawk_x, hawk_x, 2);
        }
        {  // lu, n = 33
            Real* const hawk_a = wout_tm1_a.data() + static_cast<std::size_t>(hawk_lane) * 1089;
            std::int32_t* const hawk_info = wout_tm1_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            std::int32_t* const hawk_piv = wout_tm1_piv.data() + static_cast<std::size_t>(hawk_lane) * 33;
            const auto hawk_f = hk::linalg::team::TeamLu<Real, 33>{hawk_a, hawk_piv, hawk_info};
            hk::linalg::team::lu<33>(hawk_tm, hawk_f, hawk_a);
        }
        {  // lu_det, n = 33
            Real* const hawk_a = wout_tm1_a.data() + static_cast<std::size_t>(hawk_lane) * 1089;
            std::int32_t* const hawk_info = wout_tm1_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            std::int32_t* const hawk_piv = wout_tm1_piv.data() + static_cast<std::size_t>(hawk_lane) * 33;
            Real* const hawk_x = wout_tm1_d0.data() + static_cast<std::size_t>(hawk_lane) * 1;
            const auto hawk_f = hk::linalg::team::TeamLu<Real, 33>{hawk_a, hawk_piv, hawk_info};
            if (hawk_tm.rank == 0) *hawk_x = hk::linalg::team::luDet<33>(hawk_f);
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__team_lu_33_3 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__team_lu_33_3 = 0u;
extern "C" __global__ void __launch_bounds__(256) team_lu_33_3(
    hk::abi::GRefMirror p_mut_X,
    hk::abi::ScalarHandle p_mut_det,
    hk::abi::ScalarHandle p_mut_info,
    hk::abi::GRefMirror p_mut_x,
    hk::abi::ScalarHandle p_lut_tm0_info,
    hk::abi::ScalarHandle p_lut_tm0_x0,
    hk::abi::ScalarHandle p_lut_tm0_x1,
    hk::abi::ScalarHandle p_lut_tm1_d0,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::MatOut<Real, 33, 2> mut_X(p_mut_X);
    (void)mut_X;
    const hk::ScalarOut<Real> mut_det(p_mut_det);
    (void)mut_det;
    const hk::ScalarOut<std::int32_t> mut_info(p_mut_info);
    (void)mut_info;
    const hk::VecOut<Real, 33> mut_x(p_mut_x);
    (void)mut_x;
    const hk::ScalarIn<std::int32_t> lut_tm0_info(p_lut_tm0_info);
    (void)lut_tm0_info;
    const hk::ScalarIn<Real> lut_tm0_x0(p_lut_tm0_x0);
    (void)lut_tm0_x0;
    const hk::ScalarIn<Real> lut_tm0_x1(p_lut_tm0_x1);
    (void)lut_tm0_x1;
    const hk::ScalarIn<Real> lut_tm1_d0(p_lut_tm1_d0);
    (void)lut_tm1_d0;
    __shared__ __align__(16) unsigned char hk_tile[32 * 33 * 8];
    const long long hk_lane_tiles = (count + 31) / 32;
    const long long hk_end0 = hk_lane_tiles * 2;
    const long long hk_end1 = hk_end0 + hk_lane_tiles * 3;
    const long long hk_end2 = hk_end1 + hk_lane_tiles * 1;
    const long long hk_end3 = hk_end2 + hk_lane_tiles * 1;
    for (long long hk_t = blockIdx.x; hk_t < hk_end3; hk_t += gridDim.x) {
        if (hk_t < hk_end0) hk::linalg::team::copyOutTile(lut_tm0_x0.data(), mut_x.data(), mut_x.pitch, 33LL, base, count, hk_t, hk_tile);
        else if (hk_t < hk_end1) hk::linalg::team::copyOutTile(lut_tm0_x1.data(), mut_X.data(), mut_X.pitch, 66LL, base, count, hk_t - hk_end0, hk_tile);
        else if (hk_t < hk_end2) hk::linalg::team::copyOutTile(lut_tm1_d0.data(), mut_det.data(), 0ull, 1LL, base, count, hk_t - hk_end1, hk_tile);
        else hk::linalg::team::copyOutTile(lut_tm0_info.data(), mut_info.data(), 0ull, 1LL, base, count, hk_t - hk_end2, hk_tile);
    }
    (void)nSamples;
}
