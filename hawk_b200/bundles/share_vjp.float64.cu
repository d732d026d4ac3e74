// hawk_b200 unit 'share_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) share_vjp(
    hk::abi::ScalarHandle p_aout_cut0,
    hk::abi::ScalarHandle p_aout_cut0_comp,
    hk::abi::ScalarHandle p_psc_x,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_cut0(p_aout_cut0);
    (void)aout_cut0;
    const hk::ScalarOut<Real> aout_cut0_comp(p_aout_cut0_comp);
    (void)aout_cut0_comp;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const long long hawk_rows = (count + 31) >> 5;
    for (long long hawk_r0 = hk::warp_first() * 32; hawk_r0 < hawk_rows; hawk_r0 += hk::warp_step() * 32) {
        Real hawk_terms[32];
#pragma unroll
        for (int hawk_k = 0; hawk_k < 32; ++hawk_k) hawk_terms[hawk_k] = hk::ss::identity<Real>(hk::ss::kSum);
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
                aout_cut0.data()[hawk_row] = hawk_s;
                aout_cut0_comp.data()[hawk_row] = hawk_c;
            }
        };
        hk::ss::rows_reduce<32, 1, hk::ss::kSum>(hawk_terms, hawk_ss_store);
    }
}

extern "C" __global__ void __launch_bounds__(256) share_vjp_2(
    hk::abi::ScalarHandle p_aout_cut1,
    hk::abi::ScalarHandle p_aout_cut1_comp,
    hk::abi::ScalarHandle p_psc_bar_z,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_lut_cut0,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_cut1(p_aout_cut1);
    (void)aout_cut1;
    const hk::ScalarOut<Real> aout_cut1_comp(p_aout_cut1_comp);
    (void)aout_cut1_comp;
    const hk::ScalarIn<Real> psc_bar_z(p_psc_bar_z);
    (void)psc_bar_z;
    const hk::ScalarIn<Real> psc_x(p_psc_x);
    (void)psc_x;
    const hk::ScalarIn<Real> lut_cut0(p_lut_cut0);
    (void)lut_cut0;
    const auto lut_cut0_cell = lut_cut0.cell();
    (void)lut_cut0_cell;
    const long long hawk_rows = (count + 31) >> 5;
    for (long long hawk_r0 = hk::warp_first() * 32; hawk_r0 < hawk_rows; hawk_r0 += hk::warp_step() * 32) {
        Real hawk_terms[32];
#pragma unroll
        for (int hawk_k = 0; hawk_k < 32; ++hawk_k) hawk_terms[hawk_k] = hk::ss::identity<Real>(hk::ss::kSum);
#pragma unroll
        for (int hawk_q = 0; hawk_q < 32; ++hawk_q) {
        Real* const hawk_ss = hawk_terms + hawk_q * 1;
        const long long hawk_flat = ((hawk_r0 + hawk_q) << 5) + static_cast<long long>(threadIdx.x & 31u);
        if (hawk_flat < count) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        hawk_ss[0] = (-((psc_bar_z[i].eval() * (psc_x[i].eval() / lut_cut0_cell)) / lut_cut0_cell));
        }
        }
        auto hawk_ss_store = [&](int hawk_col, auto hawk_s, auto hawk_c) {
            (void)hawk_c;
            const int hawk_q = hawk_col / 1;
            if (hawk_r0 + hawk_q >= hawk_rows) return;
            const long long hawk_row = (base >> 5) + hawk_r0 + hawk_q;
            hawk_col -= hawk_q * 1;
            if (hawk_col == 0) {
                aout_cut1.data()[hawk_row] = hawk_s;
                aout_cut1_comp.data()[hawk_row] = hawk_c;
            }
        };
        hk::ss::rows_reduce<32, 1, hk::ss::kSum>(hawk_terms, hawk_ss_store);
    }
}

extern "C" __global__ void __launch_bounds__(256) share_vjp_3(
    hk::abi::ScalarHandle p_mut_bar_x,
    hk::abi::ScalarHandle p_psc_bar_z,
    hk::abi::ScalarHandle p_lut_cut0,
    hk::abi::ScalarHandle p_lut_cut1,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_bar_x(p_mut_bar_x);
    (void)mut_bar_x;
    const hk::ScalarIn<Real> psc_bar_z(p_psc_bar_z);
    (void)psc_bar_z;
    const hk::ScalarIn<Real> lut_cut0(p_lut_cut0);
    (void)lut_cut0;
    const auto lut_cut0_cell = lut_cut0.cell();
    (void)lut_cut0_cell;
    const hk::ScalarIn<Real> lut_cut1(p_lut_cut1);
    (void)lut_cut1;
    const auto lut_cut1_cell = lut_cut1.cell();
    (void)lut_cut1_cell;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        mut_bar_x[i] = ((psc_bar_z[i].eval() / lut_cut0_cell) + lut_cut1_cell);
    }
}
