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
    // lane refill: warp w owns the spans of 64 samples at (w + k W) * 64; a lane takes
    // the next sample of its warp's span the trip its own sample leaves the loop
    Real hk_c0{};
    std::int32_t hk_c1{};
    Real hk_l0{};
    Real hk_l1{};
    const long long hk_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    const unsigned hk_lane = threadIdx.x & 31u;
    long long hk_next = hk::warp_first() * 64LL;   // the warp's next unclaimed sample
    long long hk_end = hk_next + 64LL;             // the end of its current span
    long long hk_flat = 0;
    bool hk_has = false;
    int hk_trip = 0;
    (void)nSamples;
    while (true) {
        const bool hk_needy = !hk_has;
        const unsigned hk_need = __ballot_sync(0xffffffffu, hk_needy);
        if (hk_need != 0u) {
            if (hk_next >= hk_end) {
                hk_next = hk_end + (hk_warps - 1) * 64LL;
                hk_end = hk_next + 64LL;
            }
            const long long hk_stop = hk_end < count ? hk_end : count;
            const long long hk_avail = hk_stop > hk_next ? hk_stop - hk_next : 0;
            const long long hk_rank = __popc(hk_need & ((1u << hk_lane) - 1u));
            if (hk_needy && hk_rank < hk_avail) {
                hk_flat = hk_next + hk_rank;
                const long long hawk_i = base + hk_flat;
                const hk::SampleIndex i{hawk_i};
                (void)hawk_i;
            const auto psc_M_i = psc_M[i].eval();
            const auto t2 = hawk_abi::int_from_real<std::int32_t>(static_cast<Real>(0.0));
            const auto psc_e_i = psc_e[i].eval();
                hk_c0 = psc_M_i;
                hk_c1 = t2;
                hk_l0 = psc_M_i;
                hk_l1 = psc_e_i;
                hk_trip = 0;
                hk_has = true;
            }
            const long long hk_took = __popc(hk_need);
            hk_next += hk_took < hk_avail ? hk_took : hk_avail;
        }
        if (!__any_sync(0xffffffffu, hk_has)) {
            if (hk_next >= count || (hk_next >= hk_end && hk_end + (hk_warps - 1) * 64LL >= count)) break;
            continue;
        }
        if (hk_has) {
            const long long hawk_i = base + hk_flat;
            const hk::SampleIndex i{hawk_i};
            (void)hawk_i;
            const Int hawk_k7__k = static_cast<Int>(hk_trip);
            (void)hawk_k7__k;
            const Real hawk_v7_0_Ek = hk_c0;
            const std::int32_t hawk_v7_1_n = hk_c1;
            const Real psc_M_i = hk_l0;
            const Real psc_e_i = hk_l1;
            (void)hawk_v7_0_Ek;
            (void)hawk_v7_1_n;
            (void)psc_M_i;
            (void)psc_e_i;
                const auto tb0 = (((hawk_v7_0_Ek - (psc_e_i * hk::math::sin(hawk_v7_0_Ek))) - psc_M_i) / (static_cast<Real>(1.0) - (psc_e_i * hk::math::cos(hawk_v7_0_Ek))));
                const auto tb1 = hk::math::abs(tb0);
                const Real hawk_n7_0 = (hawk_v7_0_Ek - tb0);
                const std::int32_t hawk_n7_1 = hawk_abi::int_add(hawk_v7_1_n, static_cast<std::int32_t>(1LL));
                const bool hawk_x7 = (tb1 < static_cast<Real>(1e-14));
            hk_c0 = hawk_n7_0;
            hk_c1 = hawk_n7_1;
            ++hk_trip;
            if (hawk_x7 || hk_trip >= 32) {
                const Real hawk_v7_0_Ek = hk_c0;
                const std::int32_t hawk_v7_1_n = hk_c1;
                const Real psc_M_i = hk_l0;
                const Real psc_e_i = hk_l1;
                (void)hawk_v7_0_Ek;
                (void)hawk_v7_1_n;
                (void)psc_M_i;
                (void)psc_e_i;
            mut_E[i] = hawk_v7_0_Ek;
            mut_iters[i] = hawk_v7_1_n;
                hk_has = false;
            }
        }
    }
}
