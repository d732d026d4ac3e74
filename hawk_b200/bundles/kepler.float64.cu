// hawk_b200 unit 'kepler' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) kepler(
    hk::abi::ScalarHandle p_mut_E,
    hk::abi::ScalarHandle p_mut_iters,
    hk::abi::ScalarHandle p_psc_M,
    hk::abi::ScalarHandle p_psc_e,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_E(p_mut_E);
    (void)mut_E;
    const hk::ScalarOut<std::int32_t> mut_iters(p_mut_iters);
    (void)mut_iters;
    const hk::ScalarIn<Real> psc_M(p_psc_M);
    (void)psc_M;
    const hk::ScalarIn<Real> psc_e(p_psc_e);
    (void)psc_e;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_M_i = psc_M[i].eval();
        const auto t2 = hawk_abi::int_from_real<std::int32_t>(static_cast<Real>(0.0));
        const auto psc_e_i = psc_e[i].eval();
        Real hawk_v7_0_Ek = psc_M_i;
        std::int32_t hawk_v7_1_n = t2;
        for (Int hawk_k7__k = 0; hawk_k7__k < 32; ++hawk_k7__k) {
            const auto tb0 = (((hawk_v7_0_Ek - (psc_e_i * hk::math::sin(hawk_v7_0_Ek))) - psc_M_i) / (static_cast<Real>(1.0) - (psc_e_i * hk::math::cos(hawk_v7_0_Ek))));
            const auto tb1 = hk::math::abs(tb0);
            const Real hawk_n7_0 = (hawk_v7_0_Ek - tb0);
            const std::int32_t hawk_n7_1 = hawk_abi::int_add(hawk_v7_1_n, static_cast<std::int32_t>(1LL));
            const bool hawk_x7 = (tb1 < static_cast<Real>(1e-14));
            hawk_v7_0_Ek = hawk_n7_0;
            hawk_v7_1_n = hawk_n7_1;
            if (hawk_x7) break;
        }
        mut_E[i] = hawk_v7_0_Ek;
        mut_iters[i] = hawk_v7_1_n;
    }
}
