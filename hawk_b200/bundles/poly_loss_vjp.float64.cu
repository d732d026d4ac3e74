// hawk_b200 unit 'poly_loss_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS
HK_DYNAMIC_SMEM(49280)

extern "C" __global__ void __launch_bounds__(256) poly_loss_vjp(
    hk::abi::ScalarHandle p_aout_bar_a,
    hk::abi::ScalarHandle p_aout_bar_a_comp,
    hk::abi::ScalarHandle p_aout_bar_b,
    hk::abi::ScalarHandle p_aout_bar_b_comp,
    hk::abi::ScalarHandle p_aout_bar_c,
    hk::abi::ScalarHandle p_aout_bar_c_comp,
    hk::abi::ScalarHandle p_psc_bar_r,
    hk::abi::ScalarHandle p_psc_t,
    hk::abi::ScalarHandle p_psc_x,
    hk::abi::ScalarHandle p_lut_a,
    hk::abi::ScalarHandle p_lut_b,
    hk::abi::ScalarHandle p_lut_c,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> aout_bar_a(p_aout_bar_a);
    (void)aout_bar_a;
    const hk::ScalarOut<Real> aout_bar_a_comp(p_aout_bar_a_comp);
    (void)aout_bar_a_comp;
    const hk::ScalarOut<Real> aout_bar_b(p_aout_bar_b);
    (void)aout_bar_b;
    const hk::ScalarOut<Real> aout_bar_b_comp(p_aout_bar_b_comp);
    (void)aout_bar_b_comp;
    const hk::ScalarOut<Real> aout_bar_c(p_aout_bar_c);
    (void)aout_bar_c;
    const hk::ScalarOut<Real> aout_bar_c_comp(p_aout_bar_c_comp);
    (void)aout_bar_c_comp;
    const hk::ScalarIn<Real> psc_bar_r(p_psc_bar_r, 0u);
    (void)psc_bar_r;
    const hk::ScalarIn<Real> psc_t(p_psc_t, 2048u);
    (void)psc_t;
    const hk::ScalarIn<Real> psc_x(p_psc_x, 4096u);
    (void)psc_x;
    const hk::ScalarIn<Real> lut_a(p_lut_a);
    (void)lut_a;
    const auto lut_a_cell = lut_a.cell();
    (void)lut_a_cell;
    const hk::ScalarIn<Real> lut_b(p_lut_b);
    (void)lut_b;
    const auto lut_b_cell = lut_b.cell();
    (void)lut_b_cell;
    const hk::ScalarIn<Real> lut_c(p_lut_c);
    (void)lut_c;
    const auto lut_c_cell = lut_c.cell();
    (void)lut_c_cell;
    const long long hawk_rows = (count + 31) >> 5;
    extern __shared__ __align__(128) unsigned char hk_smem[];
    hk::stage::WarpTile hk_tile(hk_smem, 6144u, 6144u);
    const bool hk_aligned = hk::stage::aligned(psc_bar_r.data(), 0ull, base * static_cast<long long>(sizeof(*psc_bar_r.data()))) && hk::stage::aligned(psc_t.data(), 0ull, base * static_cast<long long>(sizeof(*psc_t.data()))) && hk::stage::aligned(psc_x.data(), 0ull, base * static_cast<long long>(sizeof(*psc_x.data())));
    auto hk_fill = [&](long long hk_r) {      // warp-uniform: the trip starting at row hk_r
        if (!hk_aligned || ((hk_r + 8) << 5) > count) return;
        hk_tile.fill([&](unsigned char* hk_to, unsigned long long* hk_bar) {
            const long long hk_first = hk_r << 5;
            hk::stage::copy(hk_to + 0u, psc_bar_r.data() + base + hk_first, 2048u, hk_bar);
            hk::stage::copy(hk_to + 2048u, psc_t.data() + base + hk_first, 2048u, hk_bar);
            hk::stage::copy(hk_to + 4096u, psc_x.data() + base + hk_first, 2048u, hk_bar);
        });
    };
    const long long hk_step = hk::warp_step() * 8;
    long long hawk_r0 = hk::warp_first() * 8;
    if (hawk_r0 < hawk_rows) hk_fill(hawk_r0);
    for (; hawk_r0 < hawk_rows; hawk_r0 += hk_step) {
        const unsigned char* const hk_st = hk_tile.acquire();
        Real hawk_terms[24];
#pragma unroll
        for (int hawk_k = 0; hawk_k < 24; ++hawk_k) hawk_terms[hawk_k] = hk::ss::identity<Real>(hk::ss::kSum);
#pragma unroll
        for (int hawk_q = 0; hawk_q < 8; ++hawk_q) {
        Real* const hawk_ss = hawk_terms + hawk_q * 3;
        const long long hawk_flat = ((hawk_r0 + static_cast<long long>((threadIdx.x & 31u) >> 2)) << 5) + static_cast<long long>(threadIdx.x & 3u) + 4 * hawk_q;
        if (hawk_flat < count) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i, hk_st, static_cast<int>(hawk_flat - (hawk_r0 << 5))};
        (void)hawk_i;
        (void)nSamples;
        const auto psc_x_i = psc_x[i].eval();
        const auto t17 = (psc_bar_r[i].eval() * ((((((lut_a_cell * psc_x_i) * psc_x_i) * psc_x_i) + (lut_b_cell * psc_x_i)) + lut_c_cell) - psc_t[i].eval()));
        const auto t18 = (t17 + t17);
        const auto t19 = (t18 * psc_x_i);
        hawk_ss[0] = ((t19 * psc_x_i) * psc_x_i);
        hawk_ss[1] = t19;
        hawk_ss[2] = t18;
        }
        }
        if (hawk_r0 + hk_step < hawk_rows) hk_fill(hawk_r0 + hk_step);
        auto hawk_ss_store = [&](int hawk_col, auto hawk_s, auto hawk_c) {
            (void)hawk_c;
            const int hawk_q = hawk_col / 3;
            if (hawk_r0 + hawk_q >= hawk_rows) return;
            const long long hawk_row = (base >> 5) + hawk_r0 + hawk_q;
            hawk_col -= hawk_q * 3;
            if (hawk_col == 0) {
                aout_bar_a.data()[hawk_row] = hawk_s;
                aout_bar_a_comp.data()[hawk_row] = hawk_c;
            }
            else if (hawk_col == 1) {
                aout_bar_b.data()[hawk_row] = hawk_s;
                aout_bar_b_comp.data()[hawk_row] = hawk_c;
            }
            else if (hawk_col == 2) {
                aout_bar_c.data()[hawk_row] = hawk_s;
                aout_bar_c_comp.data()[hawk_row] = hawk_c;
            }
        };
        hk::ss::rows_reduce_lanes<8, 3, hk::ss::kSum>(hawk_terms, hawk_ss_store);
    }
    hk_tile.finish();
}
