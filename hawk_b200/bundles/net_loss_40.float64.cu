// hawk_b200 unit 'net_loss_40' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) net_loss_40(
    hk::abi::ScalarHandle p_aout_out,
    hk::abi::ScalarHandle p_aout_out_c,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_psc_y,
    hk::abi::ScalarHandle p_lut_W,
    hk::abi::ScalarHandle p_lut_mask,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_out(p_aout_out);
    (void)aout_out;
    const hk::ScalarOut<Real> aout_out_c(p_aout_out_c);
    (void)aout_out_c;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> psc_y(p_psc_y);
    (void)psc_y;
    const hk::ScalarIn<Real> lut_W(p_lut_W);
    (void)lut_W;
    const hk::ScalarIn<Real> lut_mask(p_lut_mask);
    (void)lut_mask;
    hk::accum::run::State hawk_run_aout_out{};
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto t2 = (static_cast<Real>(0.0) * psc_x_i);
        const auto t6 = (static_cast<Int>(hawk_i) / static_cast<Int>(40));
        const auto t12 = (hawk_abi::int_clamp_index<Int>(t6, hawk_abi::int_floordiv(static_cast<Int>(lut_mask.samples()), static_cast<Int>(8))) * static_cast<Int>(8));
        const auto t20 = (hawk_abi::int_clamp_index<Int>(t6, hawk_abi::int_floordiv(static_cast<Int>(lut_W.samples()), static_cast<Int>(24))) * static_cast<Int>(24));
        Real hawk_v25_0_pred = t2;
        for (Int hawk_k25_h = 0; hawk_k25_h < 8; ++hawk_k25_h) {
            const auto tb0 = ((lut_mask[hk::SampleIndex::make(static_cast<std::size_t>((t12 + (hawk_k25_h * static_cast<Int>(1)))))].eval() * lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t20 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k25_h) + static_cast<Int>(2)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval()) * hk::math::tanh(((lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t20 + (hawk_abi::int_clamp_index<Int>((static_cast<Int>(3) * hawk_k25_h), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval() * psc_x_i) + lut_W[hk::SampleIndex::make(static_cast<std::size_t>((t20 + (hawk_abi::int_clamp_index<Int>(((static_cast<Int>(3) * hawk_k25_h) + static_cast<Int>(1)), static_cast<Int>(24)) * static_cast<Int>(1)))))].eval())));
            const Real hawk_n25_0 = (hawk_v25_0_pred + tb0);
            hawk_v25_0_pred = hawk_n25_0;
        }
        const auto t28 = (hawk_v25_0_pred - psc_y[i].eval());
        hk::accum::run::addCompensated<8>(aout_out, aout_out_c, hk::SampleIndex::make(static_cast<std::size_t>(t6)), (t28 * t28), i, hawk_run_aout_out);
    }
}

extern "C" __global__ void __launch_bounds__(256) net_loss_40__fold_out(
    hk::abi::ScalarHandle p_aout_out,
    hk::abi::ScalarHandle p_aout_out_c,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_psc_y,
    hk::abi::ScalarHandle p_lut_W,
    hk::abi::ScalarHandle p_lut_mask,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_out(p_aout_out);
    (void)aout_out;
    const hk::ScalarOut<Real> aout_out_c(p_aout_out_c);
    (void)aout_out_c;
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
        hawk_abi::fold_companion(aout_out, aout_out_c, i);
    }
}
