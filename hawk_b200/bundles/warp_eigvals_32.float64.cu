// hawk_b200 unit 'warp_eigvals_32' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __device__ const unsigned int hk_team_threads__warp_eigvals_32 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__warp_eigvals_32 = 0u;
extern "C" __global__ void __launch_bounds__(256) warp_eigvals_32(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::GRefMirror p_mtx_A,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::MatIn<Real, 32, 32> mtx_A(p_mtx_A);
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
        { const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here(); for (Int hawk_lk = hawk_tm.rank; hawk_lk < 1024; hawk_lk += hawk_tm.size) wout_tm0_a.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 1024 + hawk_lk] = mtx_A[i].at(hawk_lk / 32, hawk_lk % 32); }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__warp_eigvals_32_2 = 32u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__warp_eigvals_32_2 = 9088u;
extern "C" __global__ void __launch_bounds__(32) warp_eigvals_32_2(
    hk::abi::ScalarHandle p_wout_tm0_a,
    hk::abi::ScalarHandle p_wout_tm0_info,
    hk::abi::ScalarHandle p_wout_tm0_w,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tm0_a(p_wout_tm0_a);
    (void)wout_tm0_a;
    const hk::ScalarOut<std::int32_t> wout_tm0_info(p_wout_tm0_info);
    (void)wout_tm0_info;
    const hk::ScalarOut<Real> wout_tm0_w(p_wout_tm0_w);
    (void)wout_tm0_w;
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
        {  // eigh_warp, n = 32
            Real* const hawk_a = wout_tm0_a.data() + static_cast<std::size_t>(hawk_lane) * 1024;
            std::int32_t* const hawk_info = wout_tm0_info.data() + static_cast<std::size_t>(hawk_lane) * 1;
            Real* const hawk_w = wout_tm0_w.data() + static_cast<std::size_t>(hawk_lane) * 32;
#if defined(__CUDA_ARCH__)
            __shared__ hk::linalg::warp::EighValuesScratch<Real> hawk_scratch;
            if (hawk_tm.rank < 32) {
                const auto hawk_r = hk::linalg::warp::eighValues<32>(hawk_scratch, static_cast<const Real*>(hawk_a));
                hawk_w[hawk_tm.rank] = hawk_r.w;
                if (hawk_tm.rank == 0) *hawk_info = hawk_r.info;
            }
#else       // the host's team of one: the one-thread form, same bits
            hk::linalg::EighValues<Real, 32> hawk_r;
            hk::linalg::eighValues<32>(hawk_r, static_cast<const Real*>(hawk_a));
            for (int hawk_k = 0; hawk_k < 32; ++hawk_k) hawk_w[hawk_k] = hawk_r.w[hawk_k];
            *hawk_info = hawk_r.info;
#endif
            hawk_tm.sync();
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__warp_eigvals_32_3 = 256u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__warp_eigvals_32_3 = 0u;
extern "C" __global__ void __launch_bounds__(256) warp_eigvals_32_3(
    hk::abi::ScalarHandle p_mut_info,
    hk::abi::GRefMirror p_mut_w,
    hk::abi::ScalarHandle p_lut_tm0_info,
    hk::abi::ScalarHandle p_lut_tm0_w,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<std::int32_t> mut_info(p_mut_info);
    (void)mut_info;
    const hk::VecOut<Real, 32> mut_w(p_mut_w);
    (void)mut_w;
    const hk::ScalarIn<std::int32_t> lut_tm0_info(p_lut_tm0_info);
    (void)lut_tm0_info;
    const hk::ScalarIn<Real> lut_tm0_w(p_lut_tm0_w);
    (void)lut_tm0_w;
    __shared__ __align__(16) unsigned char hk_tile[32 * 33 * 8];
    const long long hk_lane_tiles = (count + 31) / 32;
    const long long hk_end0 = hk_lane_tiles * 1;
    const long long hk_end1 = hk_end0 + hk_lane_tiles * 1;
    for (long long hk_t = blockIdx.x; hk_t < hk_end1; hk_t += gridDim.x) {
        if (hk_t < hk_end0) hk::linalg::team::copyOutTile(lut_tm0_w.data(), mut_w.data(), mut_w.pitch, 32LL, base, count, hk_t, hk_tile);
        else hk::linalg::team::copyOutTile(lut_tm0_info.data(), mut_info.data(), 0ull, 1LL, base, count, hk_t - hk_end0, hk_tile);
    }
    (void)nSamples;
}
