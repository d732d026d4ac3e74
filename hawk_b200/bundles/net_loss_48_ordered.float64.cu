// hawk_b200 unit 'net_loss_48_ordered' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) net_loss_48_ordered(
    hk::abi::ScalarHandle p_wout_tmb0_u,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_psc_y,
    hk::abi::ScalarHandle p_lut_W,
    hk::abi::ScalarHandle p_lut_mask,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tmb0_u(p_wout_tmb0_u);
    (void)wout_tmb0_u;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> psc_y(p_psc_y);
    (void)psc_y;
    const hk::ScalarIn<Real> lut_W(p_lut_W);
    (void)lut_W;
    const hk::ScalarIn<Real> lut_mask(p_lut_mask);
    (void)lut_mask;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto t2 = (static_cast<Real>(0.0) * psc_x_i);
        const auto t6 = (static_cast<Int>(hawk_i) / static_cast<Int>(48));
        const auto t12 = (hawk_abi::int_clamp_index<Int>(t6, hawk_abi::int_floordiv(static_cast<Int>(lut_mask.samples()), static_cast<Int>(8))) * static_cast<Int>(8));
        const auto t20 = (hawk_abi::int_clamp_index<Int>(t6, hawk_abi::int_floordiv(static_cast<Int>(lut_W.samples()), static_cast<Int>(24))) * static_cast<Int>(24));
        Real hawk_v25_0_pred = t2;
        for (Int hawk_k25_h = 0; hawk_k25_h < 8; ++hawk_k25_h) {
            const auto tb0 = ((lut_mask[hk::SampleIndex::make(static_cast<std::size_t>((t12 + (hawk_k25_h * static_cast<Int>(1)))))].eval() * lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t20 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k25_h) + static_cast<Int>(2)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval()) * hk::math::tanh(((lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t20 + (hawk_abi::int_clamp_index<Int>((static_cast<Int>(3) * hawk_k25_h), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval() * psc_x_i) + lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t20 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k25_h) + static_cast<Int>(1)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval())));
            const Real hawk_n25_0 = (hawk_v25_0_pred + tb0);
            hawk_v25_0_pred = hawk_n25_0;
        }
        const auto t28 = (hawk_v25_0_pred - psc_y[i].eval());
        wout_tmb0_u.data()[static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 1] = (t28 * t28);
    }
}

extern "C" __device__ const unsigned int hk_team_threads__net_loss_48_ordered_2 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__net_loss_48_ordered_2 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__net_loss_48_ordered_2 = 176u;
extern "C" __global__ void __launch_bounds__(32) net_loss_48_ordered_2(
    hk::abi::ScalarHandle p_wout_tmb0_gp,
    hk::abi::ScalarHandle p_wout_tmb0_u,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tmb0_gp(p_wout_tmb0_gp);
    (void)wout_tmb0_gp;
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
        {  // block_part, n = 1
            const std::size_t hawk_key = static_cast<std::size_t>(hawk_lane) / 64;
            const std::size_t hawk_grp = static_cast<std::size_t>(hawk_lane) % 64;
            const std::size_t hawk_keys = static_cast<std::size_t>(count) / 64;
            const std::size_t hawk_rows = static_cast<std::size_t>(nSamples) / hawk_keys;
            const Real* const hawk_u = wout_tmb0_u.data() + hawk_key * hawk_rows;
            #if defined(__CUDA_ARCH__)
            __shared__ Real hawk_sh[1024];
            #else
            Real hawk_sh[1024];
            #endif
            #if defined(__CUDA_ARCH__)
            hk::linalg::team::orderedPart<Real>(hawk_tm, hawk_u, hawk_rows, hawk_grp, hawk_sh);
            #else
            for (std::size_t hawk_t = 0; hawk_t < 1024; ++hawk_t) hawk_sh[hawk_t] = Real(0);
            for (std::size_t hawk_b = hawk_grp * 1024; hawk_b < hawk_rows; hawk_b += 65536) {
                const std::size_t hawk_m = hawk_rows - hawk_b < 1024 ? hawk_rows - hawk_b : 1024;
                for (std::size_t hawk_t = 0; hawk_t < hawk_m; ++hawk_t) {
                    const std::size_t hawk_r = hawk_b + hawk_t;
                    hawk_sh[hawk_t] += hawk_u[hawk_r];
                }
            }
            hawk_tm.sync();
            for (std::size_t hawk_w = 512; hawk_w > 0; hawk_w >>= 1) {
                for (std::size_t hawk_i = static_cast<std::size_t>(hawk_tm.rank); hawk_i < hawk_w; hawk_i += static_cast<std::size_t>(hawk_tm.size))
                    hawk_sh[hawk_i] += hawk_sh[hawk_i + hawk_w];
                hawk_tm.sync();
            }
            #endif
            if (hawk_tm.rank == 0) wout_tmb0_gp.data()[hawk_key * 64 + hawk_grp] = hawk_sh[0];
            hawk_tm.sync();
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__net_loss_48_ordered_3 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__net_loss_48_ordered_3 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__net_loss_48_ordered_3 = 176u;
extern "C" __global__ void __launch_bounds__(32) net_loss_48_ordered_3(
    hk::abi::ScalarHandle p_wout_out,
    hk::abi::ScalarHandle p_wout_tmb0_gp,
    hk::abi::ScalarHandle p_wout_tmb0_u,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_out(p_wout_out);
    (void)wout_out;
    const hk::ScalarOut<Real> wout_tmb0_gp(p_wout_tmb0_gp);
    (void)wout_tmb0_gp;
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
        {  // block_sum, n = 1
            const std::size_t hawk_key = static_cast<std::size_t>(hawk_lane);
            const std::size_t hawk_keys = static_cast<std::size_t>(count);
            const std::size_t hawk_rows = static_cast<std::size_t>(nSamples) / hawk_keys;
            const Real* const hawk_u = wout_tmb0_u.data();
            const Real hawk_one = Real(1);
            const Real* const hawk_v = &hawk_one;
            #if defined(__CUDA_ARCH__)
            __shared__ Real hawk_sh[64];
            #else
            Real hawk_sh[64];
            #endif
            for (std::size_t hawk_i = static_cast<std::size_t>(hawk_tm.rank); hawk_i < 64; hawk_i += static_cast<std::size_t>(hawk_tm.size))
                hawk_sh[hawk_i] = wout_tmb0_gp.data()[hawk_key * 64 + hawk_i];
            hawk_tm.sync();
            for (std::size_t hawk_w = 32; hawk_w > 0; hawk_w >>= 1) {
                for (std::size_t hawk_i = static_cast<std::size_t>(hawk_tm.rank); hawk_i < hawk_w; hawk_i += static_cast<std::size_t>(hawk_tm.size))
                    hawk_sh[hawk_i] += hawk_sh[hawk_i + hawk_w];
                hawk_tm.sync();
            }
            if (hawk_tm.rank == 0) wout_out.data()[hawk_key] = hawk_sh[0];
            hawk_tm.sync();
        }
        __syncwarp();
    }
}
