// hawk_b200 unit 'ordered_hist' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) ordered_hist(
    hk::abi::ScalarHandle p_wout_tms_acc_k,
    hk::abi::ScalarHandle p_wout_tms_acc_v,
    hk::abi::ScalarHandle p_psc_key,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<std::int32_t> wout_tms_acc_k(p_wout_tms_acc_k);
    (void)wout_tms_acc_k;
    const hk::ScalarOut<Real> wout_tms_acc_v(p_wout_tms_acc_v);
    (void)wout_tms_acc_v;
    const hk::ScalarIn<std::int32_t> psc_key(p_psc_key);
    (void)psc_key;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto t7 = ((static_cast<Int>(hawk_i) * static_cast<Int>(1)) + static_cast<Int>(0));
        wout_tms_acc_k.data()[static_cast<std::size_t>(t7) * 1] = static_cast<std::int32_t>(static_cast<Int>(psc_key[i].eval()));
        wout_tms_acc_v.data()[static_cast<std::size_t>(t7) * 1] = psc_x[i].eval();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__ordered_hist_2 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__ordered_hist_2 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__ordered_hist_2 = 160u;
extern "C" __global__ void __launch_bounds__(32) ordered_hist_2(
    hk::abi::ScalarHandle p_wout_tms_acc_m,
    hk::abi::ScalarHandle p_wout_tms_acc_p,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<std::int32_t> wout_tms_acc_m(p_wout_tms_acc_m);
    (void)wout_tms_acc_m;
    const hk::ScalarOut<Real> wout_tms_acc_p(p_wout_tms_acc_p);
    (void)wout_tms_acc_p;
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
        {  // scatter_zero, n = 1
            const std::size_t hawk_cells = static_cast<std::size_t>(count);
            const std::size_t hawk_fit = static_cast<std::size_t>(nSamples) / hawk_cells;
            const std::size_t hawk_chunks = hawk_fit < 1 ? 1 : (hawk_fit > 256 ? 256 : hawk_fit);
            Real* const hawk_p = wout_tms_acc_p.data() + static_cast<std::size_t>(hawk_lane) * hawk_chunks;
            std::int32_t* const hawk_m = const_cast<std::int32_t*>(wout_tms_acc_m.data());
            if (hawk_tm.rank == 0) {
                for (std::size_t hawk_b = 0; hawk_b < hawk_chunks; ++hawk_b) hawk_p[hawk_b] = Real(0);
                if (hawk_lane == 0) hawk_m[0] = static_cast<std::int32_t>(hawk_cells);
            }
            hawk_tm.sync();
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__ordered_hist_3 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__ordered_hist_3 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__ordered_hist_3 = 160u;
extern "C" __global__ void __launch_bounds__(32) ordered_hist_3(
    hk::abi::ScalarHandle p_wout_tms_acc_k,
    hk::abi::ScalarHandle p_wout_tms_acc_m,
    hk::abi::ScalarHandle p_wout_tms_acc_p,
    hk::abi::ScalarHandle p_wout_tms_acc_v,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<std::int32_t> wout_tms_acc_k(p_wout_tms_acc_k);
    (void)wout_tms_acc_k;
    const hk::ScalarOut<std::int32_t> wout_tms_acc_m(p_wout_tms_acc_m);
    (void)wout_tms_acc_m;
    const hk::ScalarOut<Real> wout_tms_acc_p(p_wout_tms_acc_p);
    (void)wout_tms_acc_p;
    const hk::ScalarOut<Real> wout_tms_acc_v(p_wout_tms_acc_v);
    (void)wout_tms_acc_v;
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
        {  // scatter_chunks, n = 1: 16 warps a chunk
            hk::linalg::team::scatterChunk<Real, 16>(hawk_tm, hawk_lane, count, nSamples, 1, wout_tms_acc_k.data(), wout_tms_acc_v.data(), wout_tms_acc_p.data(), const_cast<std::int32_t*>(wout_tms_acc_m.data()));
        }
        __syncwarp();
    }
}

extern "C" __device__ const unsigned int hk_team_threads__ordered_hist_4 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__ordered_hist_4 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__ordered_hist_4 = 160u;
extern "C" __global__ void __launch_bounds__(32) ordered_hist_4(
    hk::abi::ScalarHandle p_wout_acc,
    hk::abi::ScalarHandle p_wout_tms_acc_p,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_acc(p_wout_acc);
    (void)wout_acc;
    const hk::ScalarOut<Real> wout_tms_acc_p(p_wout_tms_acc_p);
    (void)wout_tms_acc_p;
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
        {  // scatter_cells, n = 1
            const std::size_t hawk_cells = static_cast<std::size_t>(count);
            const std::size_t hawk_fit = static_cast<std::size_t>(nSamples) / hawk_cells;
            const std::size_t hawk_chunks = hawk_fit < 1 ? 1 : (hawk_fit > 256 ? 256 : hawk_fit);
            const Real* const hawk_p = wout_tms_acc_p.data() + static_cast<std::size_t>(hawk_lane) * hawk_chunks;
            Real* const hawk_out = wout_acc.data();
            if (hawk_tm.rank == 0) {
                Real hawk_s = Real(0);
                for (std::size_t hawk_b = 0; hawk_b < hawk_chunks; ++hawk_b) hawk_s += hawk_p[hawk_b];
                hawk_out[hawk_lane] += hawk_s;
            }
            hawk_tm.sync();
        }
        __syncwarp();
    }
}
