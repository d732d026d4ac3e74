// hawk_b200 unit 'net_grad_40_ordered' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) net_grad_40_ordered(
    hk::abi::ScalarHandle p_wout_tmo_bar_W_i,
    hk::abi::ScalarHandle p_wout_tmo_bar_W_v,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_psc_y,
    hk::abi::ScalarHandle p_lut_W,
    hk::abi::ScalarHandle p_lut_bar_out,
    hk::abi::ScalarHandle p_lut_mask,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_tmo_bar_W_i(p_wout_tmo_bar_W_i);
    (void)wout_tmo_bar_W_i;
    const hk::ScalarOut<Real> wout_tmo_bar_W_v(p_wout_tmo_bar_W_v);
    (void)wout_tmo_bar_W_v;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> psc_y(p_psc_y);
    (void)psc_y;
    const hk::ScalarIn<Real> lut_W(p_lut_W);
    (void)lut_W;
    const hk::ScalarIn<Real> lut_bar_out(p_lut_bar_out);
    (void)lut_bar_out;
    const hk::ScalarIn<Real> lut_mask(p_lut_mask);
    (void)lut_mask;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto t4 = (static_cast<Int>(hawk_i) / static_cast<Int>(40));
        const auto psc_x_i = psc_x[i].eval();
        const auto t7 = (static_cast<Real>(0.0) * psc_x_i);
        const auto t14 = (hawk_abi::int_clamp_index<Int>(t4, hawk_abi::int_floordiv(static_cast<Int>(lut_mask.samples()), static_cast<Int>(8))) * static_cast<Int>(8));
        const auto t22 = (hawk_abi::int_clamp_index<Int>(t4, hawk_abi::int_floordiv(static_cast<Int>(lut_W.samples()), static_cast<Int>(24))) * static_cast<Int>(24));
        Real hawk_v27_0_pred = t7;
        for (Int hawk_k27_h = 0; hawk_k27_h < 8; ++hawk_k27_h) {
            const auto tb0 = ((lut_mask[hk::SampleIndex::make(static_cast<std::size_t>((t14 + (hawk_k27_h * static_cast<Int>(1)))))].eval() * lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k27_h) + static_cast<Int>(2)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval()) * hk::math::tanh(((lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>((static_cast<Int>(3) * hawk_k27_h), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval() * psc_x_i) + lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k27_h) + static_cast<Int>(1)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval())));
            const Real hawk_n27_0 = (hawk_v27_0_pred + tb0);
            hawk_v27_0_pred = hawk_n27_0;
        }
        const auto t31 = (lut_bar_out[hk::SampleIndex::make(static_cast<std::size_t>(t4))].eval() * (hawk_v27_0_pred - psc_y[i].eval()));
        const auto t32 = (t31 + t31);
        const auto t36 = (static_cast<Int>(static_cast<Int>(hawk_i)) * static_cast<Int>(24));
        const auto t38 = (t4 * static_cast<Int>(24));
        Real hawk_v40_0_bar_x = static_cast<Real>(0.0);
        for (Int hawk_k40_h = 0; hawk_k40_h < 8; ++hawk_k40_h) {
            const auto tb1 = lut_mask[hk::SampleIndex::make(static_cast<std::size_t>((t14 + (hawk_k40_h * static_cast<Int>(1)))))].eval();
            const auto tb2 = (t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k40_h) + static_cast<Int>(2)), static_cast<Int>(24)) * static_cast<Int>(1)));
            const auto tb3 = (t22 + (hawk_abi::int_clamp_index<Int>((static_cast<Int>(3) * hawk_k40_h), static_cast<Int>(24)) * static_cast<Int>(1)));
            const auto tb4 = lut_W[hk::SampleIndex::make(static_cast<std::size_t>(tb3))].eval();
            const auto tb5 = (t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k40_h) + static_cast<Int>(1)), static_cast<Int>(24)) * static_cast<Int>(1)));
            const auto tb6 = hk::math::tanh(((tb4 * psc_x_i) + lut_W[hk::SampleIndex::make(static_cast<std::size_t>(tb5))].eval()));
            const auto tb7 = ((t32 * (tb1 * lut_W[hk::SampleIndex::make(static_cast<std::size_t>(tb2))].eval())) * (static_cast<Real>(1.0) - (tb6 * tb6)));
            const auto tb8 = (tb7 * tb4);
            const auto tb9 = (static_cast<Int>(0) + ((hawk_k40_h - static_cast<Int>(0)) * static_cast<Int>(1)));
            const auto tb10 = (static_cast<Int>(8) + ((hawk_k40_h - static_cast<Int>(0)) * static_cast<Int>(1)));
            const auto tb11 = (static_cast<Int>(16) + ((hawk_k40_h - static_cast<Int>(0)) * static_cast<Int>(1)));
            wout_tmo_bar_W_v.data()[static_cast<std::size_t>((t36 + tb9)) * 1] = tb7;
            wout_tmo_bar_W_i.data()[static_cast<std::size_t>((t38 + tb9)) * 1] = static_cast<Real>(tb5);
            wout_tmo_bar_W_v.data()[static_cast<std::size_t>((t36 + tb10)) * 1] = (tb7 * psc_x_i);
            wout_tmo_bar_W_i.data()[static_cast<std::size_t>((t38 + tb10)) * 1] = static_cast<Real>(tb3);
            wout_tmo_bar_W_v.data()[static_cast<std::size_t>((t36 + tb11)) * 1] = ((t32 * tb6) * tb1);
            wout_tmo_bar_W_i.data()[static_cast<std::size_t>((t38 + tb11)) * 1] = static_cast<Real>(tb2);
            const Real hawk_n40_0 = (hawk_v40_0_bar_x + tb8);
            hawk_v40_0_bar_x = hawk_n40_0;
        }
    }
}

extern "C" __device__ const unsigned int hk_team_threads__net_grad_40_ordered_2 = 32u;
extern "C" __device__ const unsigned int hk_team_spans_run__net_grad_40_ordered_2 = 1u;
extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__net_grad_40_ordered_2 = 5120u;
extern "C" __global__ void __launch_bounds__(32) net_grad_40_ordered_2(
    hk::abi::ScalarHandle p_wout_bar_W,
    hk::abi::ScalarHandle p_wout_tmo_bar_W_i,
    hk::abi::ScalarHandle p_wout_tmo_bar_W_v,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> wout_bar_W(p_wout_bar_W);
    (void)wout_bar_W;
    const hk::ScalarOut<Real> wout_tmo_bar_W_i(p_wout_tmo_bar_W_i);
    (void)wout_tmo_bar_W_i;
    const hk::ScalarOut<Real> wout_tmo_bar_W_v(p_wout_tmo_bar_W_v);
    (void)wout_tmo_bar_W_v;
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
        {  // ordered_fold, n = 24
            const std::size_t hawk_key = static_cast<std::size_t>(hawk_lane);
            const std::size_t hawk_rows = static_cast<std::size_t>(nSamples) / static_cast<std::size_t>(count);
            const Real* const hawk_v = wout_tmo_bar_W_v.data();
            const Real* const hawk_c = wout_tmo_bar_W_i.data();
            Real* const hawk_out = wout_bar_W.data();
            for (std::size_t hawk_e = static_cast<std::size_t>(hawk_tm.rank); hawk_e < 24; hawk_e += static_cast<std::size_t>(hawk_tm.size)) {
                Real hawk_s = Real(0);
                for (std::size_t hawk_r = 0; hawk_r < hawk_rows; ++hawk_r)
                    hawk_s += hawk_v[(hawk_key * hawk_rows + hawk_r) * 24 + hawk_e];
                hawk_out[static_cast<std::size_t>(hawk_c[hawk_key * 24 + hawk_e])] = hawk_s;
            }
            hawk_tm.sync();
        }
        __syncwarp();
    }
}
