// hawk_b200 unit 'band_max' (scalar mode banded), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) band_max(
    hk::abi::ScalarHandle p_aout_hi,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_hi(p_aout_hi);
    (void)aout_hi;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const long long hawk_rows = (count + 31) >> 5;
    for (long long hawk_r0 = hk::warp_first() * 32; hawk_r0 < hawk_rows; hawk_r0 += hk::warp_step() * 32) {
        Real hawk_terms[32];
#pragma unroll
        for (int hawk_k = 0; hawk_k < 32; ++hawk_k) hawk_terms[hawk_k] = hk::ss::identity<Real>(hk::ss::kMax);
#pragma unroll
        for (int hawk_q = 0; hawk_q < 32; ++hawk_q) {
        Real* const hawk_ss = hawk_terms + hawk_q * 1;
        const long long hawk_flat = ((hawk_r0 + hawk_q) << 5) + static_cast<long long>(threadIdx.x & 31u);
        if (hawk_flat < count) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        hawk_ss[0] = psc_x[i].eval();
        }
        }
        auto hawk_ss_store = [&](int hawk_col, auto hawk_s, auto hawk_c) {
            (void)hawk_c;
            const int hawk_q = hawk_col / 1;
            if (hawk_r0 + hawk_q >= hawk_rows) return;
            const long long hawk_row = (base >> 5) + hawk_r0 + hawk_q;
            hawk_col -= hawk_q * 1;
            if (hawk_col == 0) {
                aout_hi.data()[hawk_row] = hawk_s;
            }
        };
        hk::ss::rows_reduce<32, 1, hk::ss::kMax>(hawk_terms, hawk_ss_store);
    }
}
