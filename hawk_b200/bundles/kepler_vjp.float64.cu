// hawk_b200 unit 'kepler_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) kepler_vjp(
    hk::abi::ScalarHandle p_mut_bar_M,
    hk::abi::ScalarHandle p_mut_bar_e,
    hk::abi::ScalarHandle p_psc_M,
    hk::abi::ScalarHandle p_psc_bar_E,
    hk::abi::ScalarHandle p_psc_e,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_bar_M(p_mut_bar_M);
    (void)mut_bar_M;
    const hk::ScalarOut<Real> mut_bar_e(p_mut_bar_e);
    (void)mut_bar_e;
    const hk::ScalarIn<Real> psc_M(p_psc_M);
    (void)psc_M;
    const hk::ScalarIn<Real> psc_bar_E(p_psc_bar_E);
    (void)psc_bar_E;
    const hk::ScalarIn<Real> psc_e(p_psc_e);
    (void)psc_e;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_bar_E_i = psc_bar_E[i].eval();
        const auto psc_M_i = psc_M[i].eval();
        const auto t4 = hawk_abi::int_from_real<std::int32_t>(static_cast<Real>(0.0));
        const auto psc_e_i = psc_e[i].eval();
        Real hawk_v9_0_Ek = psc_M_i;
        std::int32_t hawk_v9_1_n = t4;
        Real hawk_tp9_0[32];
        Int hawk_c9 = 0;
        for (Int hawk_k9__k = 0; hawk_k9__k < 32; ++hawk_k9__k) {
            hawk_tp9_0[hawk_k9__k] = hawk_v9_0_Ek;
            const auto tb0 = (((hawk_v9_0_Ek - (psc_e_i * hk::math::sin(hawk_v9_0_Ek))) - psc_M_i) / (static_cast<Real>(1.0) - (psc_e_i * hk::math::cos(hawk_v9_0_Ek))));
            const auto tb1 = hk::math::abs(tb0);
            const Real hawk_n9_0 = (hawk_v9_0_Ek - tb0);
            const std::int32_t hawk_n9_1 = hawk_abi::int_add(hawk_v9_1_n, static_cast<std::int32_t>(1LL));
            const bool hawk_x9 = (tb1 < static_cast<Real>(1e-14));
            hawk_v9_0_Ek = hawk_n9_0;
            hawk_v9_1_n = hawk_n9_1;
            ++hawk_c9;
            if (hawk_x9) break;
        }
        const auto t10 = hawk_c9;
        Real hawk_v11_0_bar_Ek = psc_bar_E_i;
        std::int32_t hawk_v11_1_bar_n = static_cast<std::int32_t>(0LL);
        Real hawk_v11_2_bar_M = static_cast<Real>(0.0);
        Real hawk_v11_3_bar_e = static_cast<Real>(0.0);
        for (int hawk_k11__k = static_cast<int>(31 - (32 - t10) * 1); hawk_k11__k > static_cast<int>(-1); --hawk_k11__k) {
            const auto tb2 = (-hawk_v11_0_bar_Ek);
            const auto tb3 = hawk_tp9_0[hawk_k11__k];
            const auto tb4 = hk::math::sin(tb3);
            const auto tb5 = hk::math::cos(tb3);
            const auto tb6 = (static_cast<Real>(1.0) - (psc_e_i * tb5));
            const auto tb7 = (-(-((tb2 * (((tb3 - (psc_e_i * tb4)) - psc_M_i) / tb6)) / tb6)));
            const auto tb8 = (tb2 / tb6);
            const auto tb9 = ((hawk_v11_0_bar_Ek + ((tb7 * psc_e_i) * (-hk::math::sin(tb3)))) + tb8);
            const auto tb10 = (-tb8);
            const auto tb11 = ((tb10 * psc_e_i) * hk::math::cos(tb3));
            const auto tb12 = (-tb8);
            const auto tb13 = ((tb7 * tb5) + (tb10 * tb4));
            const Real hawk_n11_0 = (tb9 + tb11);
            const Real hawk_n11_2 = (hawk_v11_2_bar_M + tb12);
            const Real hawk_n11_3 = (hawk_v11_3_bar_e + tb13);
            hawk_v11_0_bar_Ek = hawk_n11_0;
            hawk_v11_2_bar_M = hawk_n11_2;
            hawk_v11_3_bar_e = hawk_n11_3;
        }
        mut_bar_M[i] = (hawk_v11_0_bar_Ek + hawk_v11_2_bar_M);
        mut_bar_e[i] = hawk_v11_3_bar_e;
    }
}
