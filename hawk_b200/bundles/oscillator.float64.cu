// hawk_b200 unit 'oscillator' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) oscillator(
    hk::abi::ScalarHandle p_mut_k,
    hk::abi::ScalarHandle p_mut_v,
    hk::abi::ScalarHandle p_mut_x,
    hk::abi::ScalarHandle p_psc_nstop,
    hk::abi::ScalarHandle p_psc_omega,
    hk::abi::ScalarHandle p_psc_zeta,
    hk::abi::ScalarHandle p_lut_finished_count,
    hk::abi::ScalarHandle p_lut_fused_steps,
    hk::abi::ScalarHandle p_trm_terminated,
    Real p_uni_dt,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_k(p_mut_k);
    (void)mut_k;
    const hk::ScalarOut<Real> mut_v(p_mut_v);
    (void)mut_v;
    const hk::ScalarOut<Real> mut_x(p_mut_x);
    (void)mut_x;
    const hk::ScalarIn<Real> psc_nstop(p_psc_nstop);
    (void)psc_nstop;
    const hk::ScalarIn<Real> psc_omega(p_psc_omega);
    (void)psc_omega;
    const hk::ScalarIn<Real> psc_zeta(p_psc_zeta);
    (void)psc_zeta;
    const hk::ScalarIn<std::uint32_t> lut_finished_count(p_lut_finished_count);
    (void)lut_finished_count;
    const hk::ScalarIn<Int> lut_fused_steps(p_lut_fused_steps);
    (void)lut_fused_steps;
    const hk::MaskView trm_terminated(p_trm_terminated);
    (void)trm_terminated;
    const hk::MaskView trm_terminated_w(p_trm_terminated);
    (void)trm_terminated_w;
    const Real uni_dt = p_uni_dt;
    (void)uni_dt;
    if (lut_fused_steps[hk::SampleIndex::make(0)].eval() == 1) {
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        if (!trm_terminated[i].eval()) {
            const auto mut_x_i = mut_x[i].get()();
            const auto t3 = (uni_dt * static_cast<Real>(0.16666666666666666));
            const auto mut_v_i = mut_v[i].get()();
            const auto t7 = (static_cast<Real>(0.5) * uni_dt);
            const auto psc_omega_i = psc_omega[i].eval();
            const auto t10 = (-(psc_omega_i * psc_omega_i));
            const auto t14 = ((static_cast<Real>(2.0) * psc_zeta[i].eval()) * psc_omega_i);
            const auto t16 = ((t10 * mut_x_i) - (t14 * mut_v_i));
            const auto t18 = (mut_v_i + (t7 * t16));
            const auto t23 = ((t10 * (mut_x_i + (t7 * mut_v_i))) - (t14 * t18));
            const auto t25 = (mut_v_i + (t7 * t23));
            const auto t33 = ((t10 * (mut_x_i + (t7 * t18))) - (t14 * t25));
            const auto t35 = (mut_v_i + (uni_dt * t33));
            const auto t54 = (mut_k[i].get()() + static_cast<Real>(1.0));
            mut_x[i] = (mut_x_i + (t3 * ((mut_v_i + (static_cast<Real>(2.0) * (t18 + t25))) + t35)));
            mut_v[i] = (mut_v_i + (t3 * ((t16 + (static_cast<Real>(2.0) * (t23 + t33))) + ((t10 * (mut_x_i + (uni_dt * t25))) - (t14 * t35)))));
            mut_k[i] = t54;
            if (!trm_terminated[i].eval() && (t54 >= psc_nstop[i].eval())) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
        }
    }
    } else {
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        if (!trm_terminated[i].eval()) {
            const auto mut_x_i = mut_x[i].get()();
            const auto mut_v_i = mut_v[i].get()();
            const auto mut_k_i = mut_k[i].get()();
            const auto t6 = (uni_dt * static_cast<Real>(0.16666666666666666));
            const auto t9 = (static_cast<Real>(0.5) * uni_dt);
            const auto psc_omega_i = psc_omega[i].eval();
            const auto t12 = (-(psc_omega_i * psc_omega_i));
            const auto t15 = ((static_cast<Real>(2.0) * psc_zeta[i].eval()) * psc_omega_i);
            const auto psc_nstop_i = psc_nstop[i].eval();
            const auto t20 = lut_fused_steps[hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(0)))].eval();
            const auto t22 = ((t20 < static_cast<Int>(0)) ? static_cast<Int>(0) : t20);
            Real hawk_v23_0_x = mut_x_i;
            Real hawk_v23_1_v = mut_v_i;
            Real hawk_v23_2_k = mut_k_i;
            Real hawk_v23_3_finished = static_cast<Real>(0.0);
            for (int hawk_k23_step = 0; hawk_k23_step < hawk_clamp_count(t22); ++hawk_k23_step) {
                const auto tb0 = ((t12 * hawk_v23_0_x) - (t15 * hawk_v23_1_v));
                const auto tb1 = (hawk_v23_1_v + (t9 * tb0));
                const auto tb2 = ((t12 * (hawk_v23_0_x + (t9 * hawk_v23_1_v))) - (t15 * tb1));
                const auto tb3 = (hawk_v23_1_v + (t9 * tb2));
                const auto tb4 = ((t12 * (hawk_v23_0_x + (t9 * tb1))) - (t15 * tb3));
                const auto tb5 = (hawk_v23_1_v + (uni_dt * tb4));
                const auto tb6 = (t6 * ((hawk_v23_1_v + (static_cast<Real>(2.0) * (tb1 + tb3))) + tb5));
                const auto tb7 = (t6 * ((tb0 + (static_cast<Real>(2.0) * (tb2 + tb4))) + ((t12 * (hawk_v23_0_x + (uni_dt * tb3))) - (t15 * tb5))));
                const auto tb8 = (hawk_v23_2_k + static_cast<Real>(1.0));
                const auto tb9 = (tb8 >= psc_nstop_i);
                const Real hawk_n23_0 = (hawk_v23_0_x + tb6);
                const Real hawk_n23_1 = (hawk_v23_1_v + tb7);
                const Real hawk_n23_2 = tb8;
                const Real hawk_n23_3 = (tb9 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                const bool hawk_x23 = tb9;
                hawk_v23_0_x = hawk_n23_0;
                hawk_v23_1_v = hawk_n23_1;
                hawk_v23_2_k = hawk_n23_2;
                hawk_v23_3_finished = hawk_n23_3;
                if (hawk_x23) break;
            }
            mut_x[i] = hawk_v23_0_x;
            mut_v[i] = hawk_v23_1_v;
            mut_k[i] = hawk_v23_2_k;
            if (!trm_terminated[i].eval() && (hawk_v23_3_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
        }
    }
    }
}

extern "C" __global__ void __launch_bounds__(256) oscillator_persist(
    hk::abi::ScalarHandle p_mut_k,
    hk::abi::ScalarHandle p_mut_v,
    hk::abi::ScalarHandle p_mut_x,
    hk::abi::ScalarHandle p_psc_nstop,
    hk::abi::ScalarHandle p_psc_omega,
    hk::abi::ScalarHandle p_psc_zeta,
    hk::abi::ScalarHandle p_lut_finished_count,
    hk::abi::ScalarHandle p_lut_fused_steps,
    hk::abi::ScalarHandle p_trm_terminated,
    Real p_uni_dt,
    long long base,
    long long count,
    long long nSamples,
    unsigned int* hawk_next,
    unsigned long long* hawk_util,
    unsigned int* hawk_steps,
    unsigned long long* hawk_stepsum,
    unsigned int hawk_chunk)
{
    const hk::ScalarOut<Real> mut_k(p_mut_k);
    (void)mut_k;
    const hk::ScalarOut<Real> mut_v(p_mut_v);
    (void)mut_v;
    const hk::ScalarOut<Real> mut_x(p_mut_x);
    (void)mut_x;
    const hk::ScalarIn<Real> psc_nstop(p_psc_nstop);
    (void)psc_nstop;
    const hk::ScalarIn<Real> psc_omega(p_psc_omega);
    (void)psc_omega;
    const hk::ScalarIn<Real> psc_zeta(p_psc_zeta);
    (void)psc_zeta;
    const hk::ScalarIn<std::uint32_t> lut_finished_count(p_lut_finished_count);
    (void)lut_finished_count;
    const hk::ScalarIn<Int> lut_fused_steps(p_lut_fused_steps);
    (void)lut_fused_steps;
    const hk::MaskView trm_terminated(p_trm_terminated);
    (void)trm_terminated;
    const hk::MaskView trm_terminated_w(p_trm_terminated);
    (void)trm_terminated_w;
    const Real uni_dt = p_uni_dt;
    (void)uni_dt;
    Real hk_c0{};
    Real hk_c1{};
    Real hk_c2{};
    Real hk_c3{};
    Real hk_l0{};
    Real hk_l1{};
    Real hk_l2{};
    Real hk_l3{};
    Real hk_l4{};
    bool hk_has = false;              // the lane holds a sample with trips left
    bool hk_dry = false;              // the lane's last claim fell past count
    unsigned hk_s = 0u, hk_trip = 0u, hk_budget = 0u, hk_longest = 0u, hk_fin = 0u;
    unsigned long long hk_ran = 0ull;
    const unsigned hk_lane = threadIdx.x & 31u;
    const unsigned hk_chunk = hawk_chunk != 0u ? hawk_chunk : 0xffffffffu;
    (void)nSamples;
    while (true) {
        // claim: the lanes holding no sample take the next ones, one atomic per warp
        const bool hk_needy = !hk_has && !hk_dry;
        const unsigned hk_need = __ballot_sync(0xffffffffu, hk_needy);
        if (hk_need != 0u) {
            const int hk_lead = __ffs(hk_need) - 1;
            unsigned hk_first = 0u;
            if (hk_lane == static_cast<unsigned>(hk_lead))
                hk_first = atomicAdd(hawk_next, static_cast<unsigned>(__popc(hk_need)));
            hk_first = __shfl_sync(0xffffffffu, hk_first, hk_lead);
            if (hk_needy) {
                hk_s = hk_first + static_cast<unsigned>(__popc(hk_need & ((1u << hk_lane) - 1u)));
                if (static_cast<long long>(hk_s) >= count) {
                    hk_dry = true;
                } else {
                    const hk::SampleIndex i{base + static_cast<long long>(hk_s)};
                    if (trm_terminated[i].eval()) {
                        ++hk_fin;             // finished on entry: part of the batch's count
                    } else {
                            const auto mut_x_i = mut_x[i].get()();
                            const auto mut_v_i = mut_v[i].get()();
                            const auto mut_k_i = mut_k[i].get()();
                            const auto t6 = (uni_dt * static_cast<Real>(0.16666666666666666));
                            const auto t9 = (static_cast<Real>(0.5) * uni_dt);
                            const auto psc_omega_i = psc_omega[i].eval();
                            const auto t12 = (-(psc_omega_i * psc_omega_i));
                            const auto t15 = ((static_cast<Real>(2.0) * psc_zeta[i].eval()) * psc_omega_i);
                            const auto psc_nstop_i = psc_nstop[i].eval();
                            const auto t20 = lut_fused_steps[hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(0)))].eval();
                            const auto t22 = ((t20 < static_cast<Int>(0)) ? static_cast<Int>(0) : t20);
                        hk_c0 = mut_x_i;
                        hk_c1 = mut_v_i;
                        hk_c2 = mut_k_i;
                        hk_c3 = static_cast<Real>(0.0);
                        hk_l0 = t6;
                        hk_l1 = t9;
                        hk_l2 = t12;
                        hk_l3 = t15;
                        hk_l4 = psc_nstop_i;
                        hk_budget = static_cast<unsigned>(hawk_clamp_count(t22));
                        hk_trip = 0u;
                        hk_has = true;
                        if (hk_budget == 0u) {
                            const Real hawk_v23_0_x = hk_c0;
                            const Real hawk_v23_1_v = hk_c1;
                            const Real hawk_v23_2_k = hk_c2;
                            const Real hawk_v23_3_finished = hk_c3;
                            (void)hawk_v23_0_x;
                            (void)hawk_v23_1_v;
                            (void)hawk_v23_2_k;
                            (void)hawk_v23_3_finished;
                                mut_x[i] = hawk_v23_0_x;
                            mut_v[i] = hawk_v23_1_v;
                            mut_k[i] = hawk_v23_2_k;
                            if (!trm_terminated[i].eval() && (hawk_v23_3_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; ++hk_fin; }
                            hk_longest = hk_trip > hk_longest ? hk_trip : hk_longest;
                            hk_ran += hk_trip;
                            hk_has = false;
                        }
                    }
                }
            }
        }
        // leave once no lane of the warp holds a sample or can claim one
        if (!__any_sync(0xffffffffu, hk_has || !hk_dry)) break;
        if (!__any_sync(0xffffffffu, hk_has)) continue;
        // the chunk: a lane whose sample ends writes it back and idles until the next claim
        unsigned hk_iter = 0u;
        do {
            if (hk_has) {
                const hk::SampleIndex i{base + static_cast<long long>(hk_s)};
                (void)i;
                const int hawk_k23_step = static_cast<int>(hk_trip);
                (void)hawk_k23_step;
                const Real hawk_v23_0_x = hk_c0;
                const Real hawk_v23_1_v = hk_c1;
                const Real hawk_v23_2_k = hk_c2;
                const Real hawk_v23_3_finished = hk_c3;
                const Real t6 = hk_l0;
                const Real t9 = hk_l1;
                const Real t12 = hk_l2;
                const Real t15 = hk_l3;
                const Real psc_nstop_i = hk_l4;
                (void)t6;
                (void)t9;
                (void)t12;
                (void)t15;
                (void)psc_nstop_i;
                                const auto tb0 = ((t12 * hawk_v23_0_x) - (t15 * hawk_v23_1_v));
                                const auto tb1 = (hawk_v23_1_v + (t9 * tb0));
                                const auto tb2 = ((t12 * (hawk_v23_0_x + (t9 * hawk_v23_1_v))) - (t15 * tb1));
                                const auto tb3 = (hawk_v23_1_v + (t9 * tb2));
                                const auto tb4 = ((t12 * (hawk_v23_0_x + (t9 * tb1))) - (t15 * tb3));
                                const auto tb5 = (hawk_v23_1_v + (uni_dt * tb4));
                                const auto tb6 = (t6 * ((hawk_v23_1_v + (static_cast<Real>(2.0) * (tb1 + tb3))) + tb5));
                                const auto tb7 = (t6 * ((tb0 + (static_cast<Real>(2.0) * (tb2 + tb4))) + ((t12 * (hawk_v23_0_x + (uni_dt * tb3))) - (t15 * tb5))));
                                const auto tb8 = (hawk_v23_2_k + static_cast<Real>(1.0));
                                const auto tb9 = (tb8 >= psc_nstop_i);
                                const Real hawk_n23_0 = (hawk_v23_0_x + tb6);
                                const Real hawk_n23_1 = (hawk_v23_1_v + tb7);
                                const Real hawk_n23_2 = tb8;
                                const Real hawk_n23_3 = (tb9 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                                const bool hawk_x23 = tb9;
                hk_c0 = hawk_n23_0;
                hk_c1 = hawk_n23_1;
                hk_c2 = hawk_n23_2;
                hk_c3 = hawk_n23_3;
                ++hk_trip;
                if (hawk_x23 || hk_trip >= hk_budget) {
                    const Real hawk_v23_0_x = hk_c0;
                    const Real hawk_v23_1_v = hk_c1;
                    const Real hawk_v23_2_k = hk_c2;
                    const Real hawk_v23_3_finished = hk_c3;
                    (void)hawk_v23_0_x;
                    (void)hawk_v23_1_v;
                    (void)hawk_v23_2_k;
                    (void)hawk_v23_3_finished;
                        mut_x[i] = hawk_v23_0_x;
                            mut_v[i] = hawk_v23_1_v;
                            mut_k[i] = hawk_v23_2_k;
                            if (!trm_terminated[i].eval() && (hawk_v23_3_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; ++hk_fin; }
                    hk_longest = hk_trip > hk_longest ? hk_trip : hk_longest;
                    hk_ran += hk_trip;
                    hk_has = false;
                }
            }
            ++hk_iter;
        } while (hk_iter < hk_chunk && __any_sync(0xffffffffu, hk_has));
        if (hawk_util != nullptr && hk_lane == 0u) atomicAdd(&hawk_util[1], 32ull * hk_iter);
    }
    // one report per warp: the longest trip count, the steps run, the finished count
    hk::persist_report(hawk_steps, hawk_stepsum, hawk_util, hk_longest, hk_ran);
    hk::persist_finished(lut_finished_count, hk_fin);
}

extern "C" __global__ void __launch_bounds__(256) oscillator_range(
    hk::abi::ScalarHandle p_mut_k,
    hk::abi::ScalarHandle p_mut_v,
    hk::abi::ScalarHandle p_mut_x,
    hk::abi::ScalarHandle p_psc_nstop,
    hk::abi::ScalarHandle p_psc_omega,
    hk::abi::ScalarHandle p_psc_zeta,
    hk::abi::ScalarHandle p_lut_finished_count,
    hk::abi::ScalarHandle p_lut_fused_steps,
    hk::abi::ScalarHandle p_trm_terminated,
    Real p_uni_dt,
    long long base,
    long long count,
    long long nSamples,
    unsigned int* hawk_steps,
    unsigned long long* hawk_stepsum)
{
    const hk::ScalarOut<Real> mut_k(p_mut_k);
    (void)mut_k;
    const hk::ScalarOut<Real> mut_v(p_mut_v);
    (void)mut_v;
    const hk::ScalarOut<Real> mut_x(p_mut_x);
    (void)mut_x;
    const hk::ScalarIn<Real> psc_nstop(p_psc_nstop);
    (void)psc_nstop;
    const hk::ScalarIn<Real> psc_omega(p_psc_omega);
    (void)psc_omega;
    const hk::ScalarIn<Real> psc_zeta(p_psc_zeta);
    (void)psc_zeta;
    const hk::ScalarIn<std::uint32_t> lut_finished_count(p_lut_finished_count);
    (void)lut_finished_count;
    const hk::ScalarIn<Int> lut_fused_steps(p_lut_fused_steps);
    (void)lut_fused_steps;
    const hk::MaskView trm_terminated(p_trm_terminated);
    (void)trm_terminated;
    const hk::MaskView trm_terminated_w(p_trm_terminated);
    (void)trm_terminated_w;
    const Real uni_dt = p_uni_dt;
    (void)uni_dt;
    unsigned hk_longest = 0u;
    unsigned long long hk_ran = 0ull;
    if (lut_fused_steps[hk::SampleIndex::make(0)].eval() == 1) {
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const bool hk_live = !(trm_terminated[i].eval());
        if (!trm_terminated[i].eval()) {
            const auto mut_x_i = mut_x[i].get()();
            const auto t3 = (uni_dt * static_cast<Real>(0.16666666666666666));
            const auto mut_v_i = mut_v[i].get()();
            const auto t7 = (static_cast<Real>(0.5) * uni_dt);
            const auto psc_omega_i = psc_omega[i].eval();
            const auto t10 = (-(psc_omega_i * psc_omega_i));
            const auto t14 = ((static_cast<Real>(2.0) * psc_zeta[i].eval()) * psc_omega_i);
            const auto t16 = ((t10 * mut_x_i) - (t14 * mut_v_i));
            const auto t18 = (mut_v_i + (t7 * t16));
            const auto t23 = ((t10 * (mut_x_i + (t7 * mut_v_i))) - (t14 * t18));
            const auto t25 = (mut_v_i + (t7 * t23));
            const auto t33 = ((t10 * (mut_x_i + (t7 * t18))) - (t14 * t25));
            const auto t35 = (mut_v_i + (uni_dt * t33));
            const auto t54 = (mut_k[i].get()() + static_cast<Real>(1.0));
            mut_x[i] = (mut_x_i + (t3 * ((mut_v_i + (static_cast<Real>(2.0) * (t18 + t25))) + t35)));
            mut_v[i] = (mut_v_i + (t3 * ((t16 + (static_cast<Real>(2.0) * (t23 + t33))) + ((t10 * (mut_x_i + (uni_dt * t25))) - (t14 * t35)))));
            mut_k[i] = t54;
            if (!trm_terminated[i].eval() && (t54 >= psc_nstop[i].eval())) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
        }
        if (hk_live) {
            hk_longest = 1u;
            ++hk_ran;
        } else { hawk_abi::finish_count(lut_finished_count); }
    }
    } else {
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        if (!(trm_terminated[i].eval())) {
                const auto mut_x_i = mut_x[i].get()();
                const auto mut_v_i = mut_v[i].get()();
                const auto mut_k_i = mut_k[i].get()();
                const auto t6 = (uni_dt * static_cast<Real>(0.16666666666666666));
                const auto t9 = (static_cast<Real>(0.5) * uni_dt);
                const auto psc_omega_i = psc_omega[i].eval();
                const auto t12 = (-(psc_omega_i * psc_omega_i));
                const auto t15 = ((static_cast<Real>(2.0) * psc_zeta[i].eval()) * psc_omega_i);
                const auto psc_nstop_i = psc_nstop[i].eval();
                const auto t20 = lut_fused_steps[hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(0)))].eval();
                const auto t22 = ((t20 < static_cast<Int>(0)) ? static_cast<Int>(0) : t20);
            Real hk_c0 = mut_x_i;
            Real hk_c1 = mut_v_i;
            Real hk_c2 = mut_k_i;
            Real hk_c3 = static_cast<Real>(0.0);
            const int hk_cnt = hawk_clamp_count(t22);
            unsigned hk_trip = 0u;
            if (hk_cnt > 0)
            while (true) {
                const int hawk_k23_step = static_cast<int>(hk_trip);
                (void)hawk_k23_step;
                const Real hawk_v23_0_x = hk_c0;
                const Real hawk_v23_1_v = hk_c1;
                const Real hawk_v23_2_k = hk_c2;
                const Real hawk_v23_3_finished = hk_c3;
                    const auto tb0 = ((t12 * hawk_v23_0_x) - (t15 * hawk_v23_1_v));
                    const auto tb1 = (hawk_v23_1_v + (t9 * tb0));
                    const auto tb2 = ((t12 * (hawk_v23_0_x + (t9 * hawk_v23_1_v))) - (t15 * tb1));
                    const auto tb3 = (hawk_v23_1_v + (t9 * tb2));
                    const auto tb4 = ((t12 * (hawk_v23_0_x + (t9 * tb1))) - (t15 * tb3));
                    const auto tb5 = (hawk_v23_1_v + (uni_dt * tb4));
                    const auto tb6 = (t6 * ((hawk_v23_1_v + (static_cast<Real>(2.0) * (tb1 + tb3))) + tb5));
                    const auto tb7 = (t6 * ((tb0 + (static_cast<Real>(2.0) * (tb2 + tb4))) + ((t12 * (hawk_v23_0_x + (uni_dt * tb3))) - (t15 * tb5))));
                    const auto tb8 = (hawk_v23_2_k + static_cast<Real>(1.0));
                    const auto tb9 = (tb8 >= psc_nstop_i);
                    const Real hawk_n23_0 = (hawk_v23_0_x + tb6);
                    const Real hawk_n23_1 = (hawk_v23_1_v + tb7);
                    const Real hawk_n23_2 = tb8;
                    const Real hawk_n23_3 = (tb9 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                    const bool hawk_x23 = tb9;
                hk_c0 = hawk_n23_0;
                hk_c1 = hawk_n23_1;
                hk_c2 = hawk_n23_2;
                hk_c3 = hawk_n23_3;
                ++hk_trip;
                if (hawk_x23 || hk_trip >= static_cast<unsigned>(hk_cnt)) break;
            }
            {
                const Real hawk_v23_0_x = hk_c0;
                const Real hawk_v23_1_v = hk_c1;
                const Real hawk_v23_2_k = hk_c2;
                const Real hawk_v23_3_finished = hk_c3;
                (void)hawk_v23_0_x;
                (void)hawk_v23_1_v;
                (void)hawk_v23_2_k;
                (void)hawk_v23_3_finished;
                mut_x[i] = hawk_v23_0_x;
                mut_v[i] = hawk_v23_1_v;
                mut_k[i] = hawk_v23_2_k;
                if (!trm_terminated[i].eval() && (hawk_v23_3_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
            }
            hk_longest = hk_trip > hk_longest ? hk_trip : hk_longest;
            hk_ran += hk_trip;
        } else { hawk_abi::finish_count(lut_finished_count); }
    }
    }
    // one report per warp: the longest trip count and the steps run
    hk::persist_report(hawk_steps, hawk_stepsum, nullptr, hk_longest, hk_ran);
}
