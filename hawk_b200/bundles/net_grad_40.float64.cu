// hawk_b200 unit 'net_grad_40' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) net_grad_40(
    hk::abi::ScalarHandle p_aout_bar_W,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_psc_y,
    hk::abi::ScalarHandle p_lut_W,
    hk::abi::ScalarHandle p_lut_bar_out,
    hk::abi::ScalarHandle p_lut_mask,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_bar_W(p_aout_bar_W);
    (void)aout_bar_W;
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
    hk::accum::run::State hawk_run_aout_bar_W{};
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
        Real hawk_v34_0_bar_x = static_cast<Real>(0.0);
        for (Int hawk_k34_h = 0; hawk_k34_h < 8; ++hawk_k34_h) {
            const auto tb1 = lut_mask[hk::SampleIndex::make(static_cast<std::size_t>((t14 + (hawk_k34_h * static_cast<Int>(1)))))].eval();
            const auto tb2 = lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>((static_cast<Int>(3) * hawk_k34_h), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval();
            const auto tb3 = hk::math::tanh(((tb2 * psc_x_i) + lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k34_h) + static_cast<Int>(1)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval()));
            const auto tb4 = ((t32 * (tb1 * lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k34_h) + static_cast<Int>(2)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval())) * (static_cast<Real>(1.0) - (tb3 * tb3)));
            const auto tb5 = (tb4 * tb2);
            hk::accum::run::add<8>(aout_bar_W, hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k34_h) + static_cast<Int>(1)), static_cast<Int>(24)) * static_cast<Int>(1))))), tb4, i, hawk_run_aout_bar_W);
            hk::accum::run::add<8>(aout_bar_W, hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>((static_cast<Int>(3) * hawk_k34_h), static_cast<Int>(24)) * static_cast<Int>(1))))), (tb4 * psc_x_i), i, hawk_run_aout_bar_W);
            hk::accum::run::add<8>(aout_bar_W, hk::SampleIndex::make(static_cast<std::size_t>((t22 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k34_h) + static_cast<Int>(2)), static_cast<Int>(24)) * static_cast<Int>(1))))), ((t32 * tb3) * tb1), i, hawk_run_aout_bar_W);
            const Real hawk_n34_0 = (hawk_v34_0_bar_x + tb5);
            hawk_v34_0_bar_x = hawk_n34_0;
        }
    }
}
