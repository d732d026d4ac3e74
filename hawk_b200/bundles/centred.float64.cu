// hawk_b200 unit 'centred' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) centred(
    hk::abi::ScalarHandle p_aout_cut0_0,
    hk::abi::ScalarHandle p_aout_cut0_0_comp,
    hk::abi::ScalarHandle p_aout_cut0_1,
    hk::abi::ScalarHandle p_aout_cut0_1_comp,
    hk::abi::ScalarHandle p_aout_cut0_2,
    hk::abi::ScalarHandle p_aout_cut0_2_comp,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::index_t p_nsm_n_samples,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_cut0_0(p_aout_cut0_0);
    (void)aout_cut0_0;
    const hk::ScalarOut<Real> aout_cut0_0_comp(p_aout_cut0_0_comp);
    (void)aout_cut0_0_comp;
    const hk::ScalarOut<Real> aout_cut0_1(p_aout_cut0_1);
    (void)aout_cut0_1;
    const hk::ScalarOut<Real> aout_cut0_1_comp(p_aout_cut0_1_comp);
    (void)aout_cut0_1_comp;
    const hk::ScalarOut<Real> aout_cut0_2(p_aout_cut0_2);
    (void)aout_cut0_2;
    const hk::ScalarOut<Real> aout_cut0_2_comp(p_aout_cut0_2_comp);
    (void)aout_cut0_2_comp;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::abi::index_t nsm_n_samples = p_nsm_n_samples;
    (void)nsm_n_samples;
    const long long hawk_rows = (count + 31) >> 5;
    for (long long hawk_r0 = hk::warp_first() * 8; hawk_r0 < hawk_rows; hawk_r0 += hk::warp_step() * 8) {
        Real hawk_terms[24];
#pragma unroll
        for (int hawk_k = 0; hawk_k < 24; ++hawk_k) hawk_terms[hawk_k] = hk::ss::identity<Real>(hk::ss::kSum);
#pragma unroll
        for (int hawk_q = 0; hawk_q < 8; ++hawk_q) {
        Real* const hawk_ss = hawk_terms + hawk_q * 3;
        const long long hawk_flat = ((hawk_r0 + static_cast<long long>((threadIdx.x & 31u) >> 2)) << 5) + static_cast<long long>(threadIdx.x & 3u) + 4 * hawk_q;
        if (hawk_flat < count) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto t4 = hk::Item<Real, 3>{psc_x_i, (psc_x_i * psc_x_i), (static_cast<Real>(2.0) * psc_x_i)};
        const hk::Item<Real, 3> t7 = (t4 / static_cast<Real>(static_cast<Int>(nsm_n_samples)));
        hawk_ss[0] = t7.eval<0>(i);
        hawk_ss[1] = t7.eval<1>(i);
        hawk_ss[2] = t7.eval<2>(i);
        }
        }
        auto hawk_ss_store = [&](int hawk_col, auto hawk_s, auto hawk_c) {
            (void)hawk_c;
            const int hawk_q = hawk_col / 3;
            if (hawk_r0 + hawk_q >= hawk_rows) return;
            const long long hawk_row = (base >> 5) + hawk_r0 + hawk_q;
            hawk_col -= hawk_q * 3;
            if (hawk_col == 0) {
                aout_cut0_0.data()[hawk_row] = hawk_s;
                aout_cut0_0_comp.data()[hawk_row] = hawk_c;
            }
            else if (hawk_col == 1) {
                aout_cut0_1.data()[hawk_row] = hawk_s;
                aout_cut0_1_comp.data()[hawk_row] = hawk_c;
            }
            else if (hawk_col == 2) {
                aout_cut0_2.data()[hawk_row] = hawk_s;
                aout_cut0_2_comp.data()[hawk_row] = hawk_c;
            }
        };
        hk::ss::rows_reduce_lanes<8, 3, hk::ss::kSum>(hawk_terms, hawk_ss_store);
    }
}

extern "C" __global__ void __launch_bounds__(256) centred_2(
    hk::abi::GRefMirror p_mut_z,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_lut_cut0_0,
    hk::abi::ScalarHandle p_lut_cut0_1,
    hk::abi::ScalarHandle p_lut_cut0_2,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::VecOut<Real, 3> mut_z(p_mut_z);
    (void)mut_z;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> lut_cut0_0(p_lut_cut0_0);
    (void)lut_cut0_0;
    const auto lut_cut0_0_cell = lut_cut0_0.cell();
    (void)lut_cut0_0_cell;
    const hk::ScalarIn<Real> lut_cut0_1(p_lut_cut0_1);
    (void)lut_cut0_1;
    const auto lut_cut0_1_cell = lut_cut0_1.cell();
    (void)lut_cut0_1_cell;
    const hk::ScalarIn<Real> lut_cut0_2(p_lut_cut0_2);
    (void)lut_cut0_2;
    const auto lut_cut0_2_cell = lut_cut0_2.cell();
    (void)lut_cut0_2_cell;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto t4 = hk::Item<Real, 3>{psc_x_i, (psc_x_i * psc_x_i), (static_cast<Real>(2.0) * psc_x_i)};
        const auto t12 = hk::Item<Real, 3>{lut_cut0_0_cell, lut_cut0_1_cell, lut_cut0_2_cell};
        mut_z[i] = (t4 - t12);
    }
}
