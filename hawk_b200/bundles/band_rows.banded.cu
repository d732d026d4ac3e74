// hawk_b200 unit 'band_rows' (scalar mode banded), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) band_rows(
    hk::abi::ScalarHandle p_aout_q,
    hk::abi::ScalarHandle p_aout_q_comp,
    hk::abi::ScalarHandle p_aout_s,
    hk::abi::ScalarHandle p_aout_s_comp,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_q(p_aout_q);
    (void)aout_q;
    const hk::ScalarOut<Real> aout_q_comp(p_aout_q_comp);
    (void)aout_q_comp;
    const hk::ScalarOut<Real> aout_s(p_aout_s);
    (void)aout_s;
    const hk::ScalarOut<Real> aout_s_comp(p_aout_s_comp);
    (void)aout_s_comp;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const long long hawk_rows = (count + 31) >> 5;
    for (long long hawk_r0 = hk::warp_first() * 16; hawk_r0 < hawk_rows; hawk_r0 += hk::warp_step() * 16) {
        Real hawk_terms[32];
#pragma unroll
        for (int hawk_k = 0; hawk_k < 32; ++hawk_k) hawk_terms[hawk_k] = hk::ss::identity<Real>(hk::ss::kSum);
#pragma unroll
        for (int hawk_q = 0; hawk_q < 16; ++hawk_q) {
        Real* const hawk_ss = hawk_terms + hawk_q * 2;
        const long long hawk_flat = ((hawk_r0 + hawk_q) << 5) + static_cast<long long>(threadIdx.x & 31u);
        if (hawk_flat < count) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        hawk_ss[0] = psc_x_i;
        hawk_ss[1] = (psc_x_i * psc_x_i);
        }
        }
        auto hawk_ss_store = [&](int hawk_col, auto hawk_s, auto hawk_c) {
            (void)hawk_c;
            const int hawk_q = hawk_col / 2;
            if (hawk_r0 + hawk_q >= hawk_rows) return;
            const long long hawk_row = (base >> 5) + hawk_r0 + hawk_q;
            hawk_col -= hawk_q * 2;
            if (hawk_col == 0) {
                aout_s.data()[hawk_row] = hawk_s + hawk_c;
                aout_s_comp.data()[hawk_row] = static_cast<decltype(hawk_c)>(0);
            }
            else if (hawk_col == 1) {
                aout_q.data()[hawk_row] = hawk_s + hawk_c;
                aout_q_comp.data()[hawk_row] = static_cast<decltype(hawk_c)>(0);
            }
        };
        hk::ss::rows_reduce<16, 2, hk::ss::kSum>(hawk_terms, hawk_ss_store);
    }
}
