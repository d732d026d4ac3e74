// hawk_b200 unit 'orbit' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) orbit(
    hk::abi::ScalarHandle p_mut_h,
    hk::abi::ScalarHandle p_mut_n_acc,
    hk::abi::ScalarHandle p_mut_n_rej,
    hk::abi::GRefMirror p_mut_s,
    hk::abi::ScalarHandle p_mut_t,
    hk::abi::ScalarHandle p_psc_t_end,
    hk::abi::ScalarHandle p_lut_finished_count,
    hk::abi::ScalarHandle p_lut_fused_steps,
    hk::abi::ScalarHandle p_trm_terminated,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::ScalarOut<Real> mut_h(p_mut_h);
    (void)mut_h;
    const hk::ScalarOut<Real> mut_n_acc(p_mut_n_acc);
    (void)mut_n_acc;
    const hk::ScalarOut<Real> mut_n_rej(p_mut_n_rej);
    (void)mut_n_rej;
    const hk::VecOut<Real, 6> mut_s(p_mut_s);
    (void)mut_s;
    const hk::ScalarOut<Real> mut_t(p_mut_t);
    (void)mut_t;
    const hk::ScalarIn<Real> psc_t_end(p_psc_t_end);
    (void)psc_t_end;
    const hk::ScalarIn<std::uint32_t> lut_finished_count(p_lut_finished_count);
    (void)lut_finished_count;
    const hk::ScalarIn<Int> lut_fused_steps(p_lut_fused_steps);
    (void)lut_fused_steps;
    const hk::MaskView trm_terminated(p_trm_terminated);
    (void)trm_terminated;
    const hk::MaskView trm_terminated_w(p_trm_terminated);
    (void)trm_terminated_w;
    if (lut_fused_steps[hk::SampleIndex::make(0)].eval() == 1) {
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        if (!trm_terminated[i].eval()) {
            const auto mut_h_i = mut_h[i].get()();
            const auto psc_t_end_i = psc_t_end[i].eval();
            const auto mut_t_i = mut_t[i].get()();
            const auto t3 = (psc_t_end_i - mut_t_i);
            const auto t4 = (mut_h_i >= t3);
            const auto t5 = (t4 ? t3 : mut_h_i);
            const auto t7 = (t5 * static_cast<Real>(0.04880952380952381));
            const auto mut_s_i = mut_s[i].get();
            const auto t10 = mut_s_i.eval<3>(i);
            const auto t13 = mut_s_i.eval<0>(i);
            const auto t15 = mut_s_i.eval<1>(i);
            const auto t18 = mut_s_i.eval<2>(i);
            const auto t20 = (((t13 * t13) + (t15 * t15)) + (t18 * t18));
            const auto t23 = (static_cast<Real>(1.0) / (t20 * hk::math::sqrt(t20)));
            const auto t25 = (-(t13 * t23));
            const auto t37 = (t13 + (t5 * (static_cast<Real>(0.07407407407407407) * t10)));
            const auto t39 = mut_s_i.eval<4>(i);
            const auto t42 = (t15 + (t5 * (static_cast<Real>(0.07407407407407407) * t39)));
            const auto t45 = mut_s_i.eval<5>(i);
            const auto t48 = (t18 + (t5 * (static_cast<Real>(0.07407407407407407) * t45)));
            const auto t50 = (((t37 * t37) + (t42 * t42)) + (t48 * t48));
            const auto t53 = (static_cast<Real>(1.0) / (t50 * hk::math::sqrt(t50)));
            const auto t59 = (t10 + (t5 * ((static_cast<Real>(0.027777777777777776) * t25) + (static_cast<Real>(0.08333333333333333) * (-(t37 * t53))))));
            const auto t63 = (t13 + (t5 * ((static_cast<Real>(0.041666666666666664) * t10) + (static_cast<Real>(0.125) * t59))));
            const auto t67 = (-(t15 * t23));
            const auto t74 = (t39 + (t5 * ((static_cast<Real>(0.027777777777777776) * t67) + (static_cast<Real>(0.08333333333333333) * (-(t42 * t53))))));
            const auto t78 = (t15 + (t5 * ((static_cast<Real>(0.041666666666666664) * t39) + (static_cast<Real>(0.125) * t74))));
            const auto t83 = (-(t18 * t23));
            const auto t90 = (t45 + (t5 * ((static_cast<Real>(0.027777777777777776) * t83) + (static_cast<Real>(0.08333333333333333) * (-(t48 * t53))))));
            const auto t94 = (t18 + (t5 * ((static_cast<Real>(0.041666666666666664) * t45) + (static_cast<Real>(0.125) * t90))));
            const auto t96 = (((t63 * t63) + (t78 * t78)) + (t94 * t94));
            const auto t99 = (static_cast<Real>(1.0) / (t96 * hk::math::sqrt(t96)));
            const auto t101 = (-(t63 * t99));
            const auto t102 = (static_cast<Real>(-2.0792682926829267) * t101);
            const auto t119 = (t13 + (t5 * ((static_cast<Real>(0.027777777777777776) * t10) + (static_cast<Real>(0.08333333333333333) * (t10 + (t5 * (static_cast<Real>(0.07407407407407407) * t25)))))));
            const auto t128 = (t15 + (t5 * ((static_cast<Real>(0.027777777777777776) * t39) + (static_cast<Real>(0.08333333333333333) * (t39 + (t5 * (static_cast<Real>(0.07407407407407407) * t67)))))));
            const auto t138 = (t18 + (t5 * ((static_cast<Real>(0.027777777777777776) * t45) + (static_cast<Real>(0.08333333333333333) * (t45 + (t5 * (static_cast<Real>(0.07407407407407407) * t83)))))));
            const auto t140 = (((t119 * t119) + (t128 * t128)) + (t138 * t138));
            const auto t143 = (static_cast<Real>(1.0) / (t140 * hk::math::sqrt(t140)));
            const auto t145 = (-(t119 * t143));
            const auto t149 = (t10 + (t5 * ((static_cast<Real>(0.041666666666666664) * t25) + (static_cast<Real>(0.125) * t145))));
            const auto t153 = (t13 + (t5 * (((static_cast<Real>(0.4166666666666667) * t10) + (static_cast<Real>(-1.5625) * t59)) + (static_cast<Real>(1.5625) * t149))));
            const auto t160 = (-(t128 * t143));
            const auto t164 = (t39 + (t5 * ((static_cast<Real>(0.041666666666666664) * t67) + (static_cast<Real>(0.125) * t160))));
            const auto t168 = (t15 + (t5 * (((static_cast<Real>(0.4166666666666667) * t39) + (static_cast<Real>(-1.5625) * t74)) + (static_cast<Real>(1.5625) * t164))));
            const auto t176 = (-(t138 * t143));
            const auto t180 = (t45 + (t5 * ((static_cast<Real>(0.041666666666666664) * t83) + (static_cast<Real>(0.125) * t176))));
            const auto t184 = (t18 + (t5 * (((static_cast<Real>(0.4166666666666667) * t45) + (static_cast<Real>(-1.5625) * t90)) + (static_cast<Real>(1.5625) * t180))));
            const auto t186 = (((t153 * t153) + (t168 * t168)) + (t184 * t184));
            const auto t189 = (static_cast<Real>(1.0) / (t186 * hk::math::sqrt(t186)));
            const auto t191 = (-(t153 * t189));
            const auto t192 = (static_cast<Real>(4.3863414634146345) * t191);
            const auto t207 = (t10 + (t5 * (((static_cast<Real>(0.4166666666666667) * t25) + (static_cast<Real>(-1.5625) * t145)) + (static_cast<Real>(1.5625) * t101))));
            const auto t211 = (t13 + (t5 * (((static_cast<Real>(0.05) * t10) + (static_cast<Real>(0.25) * t149)) + (static_cast<Real>(0.2) * t207))));
            const auto t220 = (-(t78 * t99));
            const auto t224 = (t39 + (t5 * (((static_cast<Real>(0.4166666666666667) * t67) + (static_cast<Real>(-1.5625) * t160)) + (static_cast<Real>(1.5625) * t220))));
            const auto t228 = (t15 + (t5 * (((static_cast<Real>(0.05) * t39) + (static_cast<Real>(0.25) * t164)) + (static_cast<Real>(0.2) * t224))));
            const auto t238 = (-(t94 * t99));
            const auto t242 = (t45 + (t5 * (((static_cast<Real>(0.4166666666666667) * t83) + (static_cast<Real>(-1.5625) * t176)) + (static_cast<Real>(1.5625) * t238))));
            const auto t246 = (t18 + (t5 * (((static_cast<Real>(0.05) * t45) + (static_cast<Real>(0.25) * t180)) + (static_cast<Real>(0.2) * t242))));
            const auto t248 = (((t211 * t211) + (t228 * t228)) + (t246 * t246));
            const auto t251 = (static_cast<Real>(1.0) / (t248 * hk::math::sqrt(t248)));
            const auto t253 = (-(t211 * t251));
            const auto t272 = (t10 + (t5 * (((static_cast<Real>(0.05) * t25) + (static_cast<Real>(0.25) * t101)) + (static_cast<Real>(0.2) * t191))));
            const auto t276 = (t13 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t10) + (static_cast<Real>(1.1574074074074074) * t149)) + (static_cast<Real>(-2.4074074074074074) * t207)) + (static_cast<Real>(2.314814814814815) * t272))));
            const auto t287 = (-(t168 * t189));
            const auto t291 = (t39 + (t5 * (((static_cast<Real>(0.05) * t67) + (static_cast<Real>(0.25) * t220)) + (static_cast<Real>(0.2) * t287))));
            const auto t295 = (t15 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t39) + (static_cast<Real>(1.1574074074074074) * t164)) + (static_cast<Real>(-2.4074074074074074) * t224)) + (static_cast<Real>(2.314814814814815) * t291))));
            const auto t307 = (-(t184 * t189));
            const auto t311 = (t45 + (t5 * (((static_cast<Real>(0.05) * t83) + (static_cast<Real>(0.25) * t238)) + (static_cast<Real>(0.2) * t307))));
            const auto t315 = (t18 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t45) + (static_cast<Real>(1.1574074074074074) * t180)) + (static_cast<Real>(-2.4074074074074074) * t242)) + (static_cast<Real>(2.314814814814815) * t311))));
            const auto t317 = (((t276 * t276) + (t295 * t295)) + (t315 * t315));
            const auto t320 = (static_cast<Real>(1.0) / (t317 * hk::math::sqrt(t317)));
            const auto t322 = (-(t276 * t320));
            const auto t343 = (t10 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t25) + (static_cast<Real>(1.1574074074074074) * t101)) + (static_cast<Real>(-2.4074074074074074) * t191)) + (static_cast<Real>(2.314814814814815) * t253))));
            const auto t347 = (t13 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t10) + (static_cast<Real>(0.27111111111111114) * t207)) + (static_cast<Real>(-0.2222222222222222) * t272)) + (static_cast<Real>(0.014444444444444444) * t343))));
            const auto t360 = (-(t228 * t251));
            const auto t364 = (t39 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t67) + (static_cast<Real>(1.1574074074074074) * t220)) + (static_cast<Real>(-2.4074074074074074) * t287)) + (static_cast<Real>(2.314814814814815) * t360))));
            const auto t368 = (t15 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t39) + (static_cast<Real>(0.27111111111111114) * t224)) + (static_cast<Real>(-0.2222222222222222) * t291)) + (static_cast<Real>(0.014444444444444444) * t364))));
            const auto t382 = (-(t246 * t251));
            const auto t386 = (t45 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t83) + (static_cast<Real>(1.1574074074074074) * t238)) + (static_cast<Real>(-2.4074074074074074) * t307)) + (static_cast<Real>(2.314814814814815) * t382))));
            const auto t390 = (t18 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t45) + (static_cast<Real>(0.27111111111111114) * t242)) + (static_cast<Real>(-0.2222222222222222) * t311)) + (static_cast<Real>(0.014444444444444444) * t386))));
            const auto t392 = (((t347 * t347) + (t368 * t368)) + (t390 * t390));
            const auto t395 = (static_cast<Real>(1.0) / (t392 * hk::math::sqrt(t392)));
            const auto t397 = (-(t347 * t395));
            const auto t424 = (t10 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t25) + (static_cast<Real>(0.27111111111111114) * t191)) + (static_cast<Real>(-0.2222222222222222) * t253)) + (static_cast<Real>(0.014444444444444444) * t322))));
            const auto t428 = (t13 + (t5 * ((((((static_cast<Real>(2.0) * t10) + (static_cast<Real>(-8.833333333333334) * t149)) + (static_cast<Real>(15.644444444444444) * t207)) + (static_cast<Real>(-11.88888888888889) * t272)) + (static_cast<Real>(0.7444444444444445) * t343)) + (static_cast<Real>(3.0) * t424))));
            const auto t445 = (-(t295 * t320));
            const auto t449 = (t39 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t67) + (static_cast<Real>(0.27111111111111114) * t287)) + (static_cast<Real>(-0.2222222222222222) * t360)) + (static_cast<Real>(0.014444444444444444) * t445))));
            const auto t453 = (t15 + (t5 * ((((((static_cast<Real>(2.0) * t39) + (static_cast<Real>(-8.833333333333334) * t164)) + (static_cast<Real>(15.644444444444444) * t224)) + (static_cast<Real>(-11.88888888888889) * t291)) + (static_cast<Real>(0.7444444444444445) * t364)) + (static_cast<Real>(3.0) * t449))));
            const auto t471 = (-(t315 * t320));
            const auto t475 = (t45 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t83) + (static_cast<Real>(0.27111111111111114) * t307)) + (static_cast<Real>(-0.2222222222222222) * t382)) + (static_cast<Real>(0.014444444444444444) * t471))));
            const auto t479 = (t18 + (t5 * ((((((static_cast<Real>(2.0) * t45) + (static_cast<Real>(-8.833333333333334) * t180)) + (static_cast<Real>(15.644444444444444) * t242)) + (static_cast<Real>(-11.88888888888889) * t311)) + (static_cast<Real>(0.7444444444444445) * t386)) + (static_cast<Real>(3.0) * t475))));
            const auto t481 = (((t428 * t428) + (t453 * t453)) + (t479 * t479));
            const auto t484 = (static_cast<Real>(1.0) / (t481 * hk::math::sqrt(t481)));
            const auto t486 = (-(t428 * t484));
            const auto t520 = (t10 + (t5 * ((((((static_cast<Real>(2.0) * t25) + (static_cast<Real>(-8.833333333333334) * t101)) + (static_cast<Real>(15.644444444444444) * t191)) + (static_cast<Real>(-11.88888888888889) * t253)) + (static_cast<Real>(0.7444444444444445) * t322)) + (static_cast<Real>(3.0) * t397))));
            const auto t524 = (t13 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t10) + (static_cast<Real>(0.21296296296296297) * t149)) + (static_cast<Real>(-7.229629629629629) * t207)) + (static_cast<Real>(5.7592592592592595) * t272)) + (static_cast<Real>(-0.31666666666666665) * t343)) + (static_cast<Real>(2.8333333333333335) * t424)) + (static_cast<Real>(-0.08333333333333333) * t520))));
            const auto t547 = (-(t368 * t395));
            const auto t551 = (t39 + (t5 * ((((((static_cast<Real>(2.0) * t67) + (static_cast<Real>(-8.833333333333334) * t220)) + (static_cast<Real>(15.644444444444444) * t287)) + (static_cast<Real>(-11.88888888888889) * t360)) + (static_cast<Real>(0.7444444444444445) * t445)) + (static_cast<Real>(3.0) * t547))));
            const auto t555 = (t15 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t39) + (static_cast<Real>(0.21296296296296297) * t164)) + (static_cast<Real>(-7.229629629629629) * t224)) + (static_cast<Real>(5.7592592592592595) * t291)) + (static_cast<Real>(-0.31666666666666665) * t364)) + (static_cast<Real>(2.8333333333333335) * t449)) + (static_cast<Real>(-0.08333333333333333) * t551))));
            const auto t579 = (-(t390 * t395));
            const auto t583 = (t45 + (t5 * ((((((static_cast<Real>(2.0) * t83) + (static_cast<Real>(-8.833333333333334) * t238)) + (static_cast<Real>(15.644444444444444) * t307)) + (static_cast<Real>(-11.88888888888889) * t382)) + (static_cast<Real>(0.7444444444444445) * t471)) + (static_cast<Real>(3.0) * t579))));
            const auto t587 = (t18 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t45) + (static_cast<Real>(0.21296296296296297) * t180)) + (static_cast<Real>(-7.229629629629629) * t242)) + (static_cast<Real>(5.7592592592592595) * t311)) + (static_cast<Real>(-0.31666666666666665) * t386)) + (static_cast<Real>(2.8333333333333335) * t475)) + (static_cast<Real>(-0.08333333333333333) * t583))));
            const auto t589 = (((t524 * t524) + (t555 * t555)) + (t587 * t587));
            const auto t592 = (static_cast<Real>(1.0) / (t589 * hk::math::sqrt(t589)));
            const auto t594 = (-(t524 * t592));
            const auto t620 = (t10 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t25) + (static_cast<Real>(-0.14634146341463414) * t253)) + (static_cast<Real>(-0.014634146341463415) * t322)) + (static_cast<Real>(-0.07317073170731707) * t397)) + (static_cast<Real>(0.07317073170731707) * t486)) + (static_cast<Real>(0.14634146341463414) * t594))));
            const auto t665 = (t10 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t25) + (static_cast<Real>(0.21296296296296297) * t101)) + (static_cast<Real>(-7.229629629629629) * t191)) + (static_cast<Real>(5.7592592592592595) * t253)) + (static_cast<Real>(-0.31666666666666665) * t322)) + (static_cast<Real>(2.8333333333333335) * t397)) + (static_cast<Real>(-0.08333333333333333) * t486))));
            const auto t669 = (t13 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t10) + (static_cast<Real>(-0.14634146341463414) * t272)) + (static_cast<Real>(-0.014634146341463415) * t343)) + (static_cast<Real>(-0.07317073170731707) * t424)) + (static_cast<Real>(0.07317073170731707) * t520)) + (static_cast<Real>(0.14634146341463414) * t665))));
            const auto t692 = (-(t453 * t484));
            const auto t696 = (t39 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t67) + (static_cast<Real>(0.21296296296296297) * t220)) + (static_cast<Real>(-7.229629629629629) * t287)) + (static_cast<Real>(5.7592592592592595) * t360)) + (static_cast<Real>(-0.31666666666666665) * t445)) + (static_cast<Real>(2.8333333333333335) * t547)) + (static_cast<Real>(-0.08333333333333333) * t692))));
            const auto t700 = (t15 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t39) + (static_cast<Real>(-0.14634146341463414) * t291)) + (static_cast<Real>(-0.014634146341463415) * t364)) + (static_cast<Real>(-0.07317073170731707) * t449)) + (static_cast<Real>(0.07317073170731707) * t551)) + (static_cast<Real>(0.14634146341463414) * t696))));
            const auto t724 = (-(t479 * t484));
            const auto t728 = (t45 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t83) + (static_cast<Real>(0.21296296296296297) * t238)) + (static_cast<Real>(-7.229629629629629) * t307)) + (static_cast<Real>(5.7592592592592595) * t382)) + (static_cast<Real>(-0.31666666666666665) * t471)) + (static_cast<Real>(2.8333333333333335) * t579)) + (static_cast<Real>(-0.08333333333333333) * t724))));
            const auto t732 = (t18 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t45) + (static_cast<Real>(-0.14634146341463414) * t311)) + (static_cast<Real>(-0.014634146341463415) * t386)) + (static_cast<Real>(-0.07317073170731707) * t475)) + (static_cast<Real>(0.07317073170731707) * t583)) + (static_cast<Real>(0.14634146341463414) * t728))));
            const auto t734 = (((t669 * t669) + (t700 * t700)) + (t732 * t732));
            const auto t737 = (static_cast<Real>(1.0) / (t734 * hk::math::sqrt(t734)));
            const auto t739 = (-(t669 * t737));
            const auto t743 = (t10 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t25) + t102) + t192) + (static_cast<Real>(-3.524390243902439) * t253)) + (static_cast<Real>(0.5348780487804878) * t322)) + (static_cast<Real>(0.6219512195121951) * t397)) + (static_cast<Real>(0.20121951219512196) * t486)) + (static_cast<Real>(0.2926829268292683) * t594)) + (static_cast<Real>(1.0) * t739))));
            const auto t766 = (t13 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t272) + (static_cast<Real>(0.2571428571428571) * t343)) + (static_cast<Real>(0.2571428571428571) * t424)) + (static_cast<Real>(0.03214285714285714) * t520)) + (static_cast<Real>(0.03214285714285714) * t665)) + (static_cast<Real>(0.04880952380952381) * t620)) + (static_cast<Real>(0.04880952380952381) * t743))));
            const auto t775 = (static_cast<Real>(-2.0792682926829267) * t220);
            const auto t777 = (static_cast<Real>(4.3863414634146345) * t287);
            const auto t788 = (-(t555 * t592));
            const auto t807 = (t39 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t67) + (static_cast<Real>(-0.14634146341463414) * t360)) + (static_cast<Real>(-0.014634146341463415) * t445)) + (static_cast<Real>(-0.07317073170731707) * t547)) + (static_cast<Real>(0.07317073170731707) * t692)) + (static_cast<Real>(0.14634146341463414) * t788))));
            const auto t824 = (-(t700 * t737));
            const auto t828 = (t39 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t67) + t775) + t777) + (static_cast<Real>(-3.524390243902439) * t360)) + (static_cast<Real>(0.5348780487804878) * t445)) + (static_cast<Real>(0.6219512195121951) * t547)) + (static_cast<Real>(0.20121951219512196) * t692)) + (static_cast<Real>(0.2926829268292683) * t788)) + (static_cast<Real>(1.0) * t824))));
            const auto t847 = (t15 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t291) + (static_cast<Real>(0.2571428571428571) * t364)) + (static_cast<Real>(0.2571428571428571) * t449)) + (static_cast<Real>(0.03214285714285714) * t551)) + (static_cast<Real>(0.03214285714285714) * t696)) + (static_cast<Real>(0.04880952380952381) * t807)) + (static_cast<Real>(0.04880952380952381) * t828))));
            const auto t857 = (static_cast<Real>(-2.0792682926829267) * t238);
            const auto t859 = (static_cast<Real>(4.3863414634146345) * t307);
            const auto t870 = (-(t587 * t592));
            const auto t889 = (t45 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t83) + (static_cast<Real>(-0.14634146341463414) * t382)) + (static_cast<Real>(-0.014634146341463415) * t471)) + (static_cast<Real>(-0.07317073170731707) * t579)) + (static_cast<Real>(0.07317073170731707) * t724)) + (static_cast<Real>(0.14634146341463414) * t870))));
            const auto t906 = (-(t732 * t737));
            const auto t910 = (t45 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t83) + t857) + t859) + (static_cast<Real>(-3.524390243902439) * t382)) + (static_cast<Real>(0.5348780487804878) * t471)) + (static_cast<Real>(0.6219512195121951) * t579)) + (static_cast<Real>(0.20121951219512196) * t724)) + (static_cast<Real>(0.2926829268292683) * t870)) + (static_cast<Real>(1.0) * t906))));
            const auto t929 = (t18 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t311) + (static_cast<Real>(0.2571428571428571) * t386)) + (static_cast<Real>(0.2571428571428571) * t475)) + (static_cast<Real>(0.03214285714285714) * t583)) + (static_cast<Real>(0.03214285714285714) * t728)) + (static_cast<Real>(0.04880952380952381) * t889)) + (static_cast<Real>(0.04880952380952381) * t910))));
            const auto t939 = (static_cast<Real>(-2.0792682926829267) * t149);
            const auto t941 = (static_cast<Real>(4.3863414634146345) * t207);
            const auto t954 = (t13 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t10) + t939) + t941) + (static_cast<Real>(-3.6707317073170733) * t272)) + (static_cast<Real>(0.5202439024390244) * t343)) + (static_cast<Real>(0.5487804878048781) * t424)) + (static_cast<Real>(0.27439024390243905) * t520)) + (static_cast<Real>(0.43902439024390244) * t665))));
            const auto t957 = (static_cast<Real>(-2.0792682926829267) * t164);
            const auto t959 = (static_cast<Real>(4.3863414634146345) * t224);
            const auto t972 = (t15 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t39) + t957) + t959) + (static_cast<Real>(-3.6707317073170733) * t291)) + (static_cast<Real>(0.5202439024390244) * t364)) + (static_cast<Real>(0.5487804878048781) * t449)) + (static_cast<Real>(0.27439024390243905) * t551)) + (static_cast<Real>(0.43902439024390244) * t696))));
            const auto t976 = (static_cast<Real>(-2.0792682926829267) * t180);
            const auto t978 = (static_cast<Real>(4.3863414634146345) * t242);
            const auto t991 = (t18 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t45) + t976) + t978) + (static_cast<Real>(-3.6707317073170733) * t311)) + (static_cast<Real>(0.5202439024390244) * t386)) + (static_cast<Real>(0.5487804878048781) * t475)) + (static_cast<Real>(0.27439024390243905) * t583)) + (static_cast<Real>(0.43902439024390244) * t728))));
            const auto t993 = (((t954 * t954) + (t972 * t972)) + (t991 * t991));
            const auto t996 = (static_cast<Real>(1.0) / (t993 * hk::math::sqrt(t993)));
            const auto t1019 = (t13 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t10) + t939) + t941) + (static_cast<Real>(-3.524390243902439) * t272)) + (static_cast<Real>(0.5348780487804878) * t343)) + (static_cast<Real>(0.6219512195121951) * t424)) + (static_cast<Real>(0.20121951219512196) * t520)) + (static_cast<Real>(0.2926829268292683) * t665)) + (static_cast<Real>(1.0) * t620))));
            const auto t1037 = (t15 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t39) + t957) + t959) + (static_cast<Real>(-3.524390243902439) * t291)) + (static_cast<Real>(0.5348780487804878) * t364)) + (static_cast<Real>(0.6219512195121951) * t449)) + (static_cast<Real>(0.20121951219512196) * t551)) + (static_cast<Real>(0.2926829268292683) * t696)) + (static_cast<Real>(1.0) * t807))));
            const auto t1056 = (t18 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t45) + t976) + t978) + (static_cast<Real>(-3.524390243902439) * t311)) + (static_cast<Real>(0.5348780487804878) * t386)) + (static_cast<Real>(0.6219512195121951) * t475)) + (static_cast<Real>(0.20121951219512196) * t583)) + (static_cast<Real>(0.2926829268292683) * t728)) + (static_cast<Real>(1.0) * t889))));
            const auto t1058 = (((t1019 * t1019) + (t1037 * t1037)) + (t1056 * t1056));
            const auto t1061 = (static_cast<Real>(1.0) / (t1058 * hk::math::sqrt(t1058)));
            const auto t1063 = (-(t1019 * t1061));
            const auto t1082 = (t10 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t253) + (static_cast<Real>(0.2571428571428571) * t322)) + (static_cast<Real>(0.2571428571428571) * t397)) + (static_cast<Real>(0.03214285714285714) * t486)) + (static_cast<Real>(0.03214285714285714) * t594)) + (static_cast<Real>(0.04880952380952381) * t739)) + (static_cast<Real>(0.04880952380952381) * t1063))));
            const auto t1098 = (-(t1037 * t1061));
            const auto t1117 = (t39 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t360) + (static_cast<Real>(0.2571428571428571) * t445)) + (static_cast<Real>(0.2571428571428571) * t547)) + (static_cast<Real>(0.03214285714285714) * t692)) + (static_cast<Real>(0.03214285714285714) * t788)) + (static_cast<Real>(0.04880952380952381) * t824)) + (static_cast<Real>(0.04880952380952381) * t1098))));
            const auto t1133 = (-(t1056 * t1061));
            const auto t1152 = (t45 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t382) + (static_cast<Real>(0.2571428571428571) * t471)) + (static_cast<Real>(0.2571428571428571) * t579)) + (static_cast<Real>(0.03214285714285714) * t724)) + (static_cast<Real>(0.03214285714285714) * t870)) + (static_cast<Real>(0.04880952380952381) * t906)) + (static_cast<Real>(0.04880952380952381) * t1133))));
            const auto t1159 = hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax((hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t10) + (static_cast<Real>(1.0) * (t10 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t25) + t102) + t192) + (static_cast<Real>(-3.6707317073170733) * t253)) + (static_cast<Real>(0.5202439024390244) * t322)) + (static_cast<Real>(0.5487804878048781) * t397)) + (static_cast<Real>(0.27439024390243905) * t486)) + (static_cast<Real>(0.43902439024390244) * t594)))))) + (static_cast<Real>(-1.0) * t620)) + (static_cast<Real>(-1.0) * t743)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t766), hk::math::abs(t13))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t39) + (static_cast<Real>(1.0) * (t39 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t67) + t775) + t777) + (static_cast<Real>(-3.6707317073170733) * t360)) + (static_cast<Real>(0.5202439024390244) * t445)) + (static_cast<Real>(0.5487804878048781) * t547)) + (static_cast<Real>(0.27439024390243905) * t692)) + (static_cast<Real>(0.43902439024390244) * t788)))))) + (static_cast<Real>(-1.0) * t807)) + (static_cast<Real>(-1.0) * t828)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t847), hk::math::abs(t15)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t45) + (static_cast<Real>(1.0) * (t45 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t83) + t857) + t859) + (static_cast<Real>(-3.6707317073170733) * t382)) + (static_cast<Real>(0.5202439024390244) * t471)) + (static_cast<Real>(0.5487804878048781) * t579)) + (static_cast<Real>(0.27439024390243905) * t724)) + (static_cast<Real>(0.43902439024390244) * t870)))))) + (static_cast<Real>(-1.0) * t889)) + (static_cast<Real>(-1.0) * t910)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t929), hk::math::abs(t18)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t25) + (static_cast<Real>(1.0) * (-(t954 * t996)))) + (static_cast<Real>(-1.0) * t739)) + (static_cast<Real>(-1.0) * t1063)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t1082), hk::math::abs(t10)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t67) + (static_cast<Real>(1.0) * (-(t972 * t996)))) + (static_cast<Real>(-1.0) * t824)) + (static_cast<Real>(-1.0) * t1098)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t1117), hk::math::abs(t39)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t83) + (static_cast<Real>(1.0) * (-(t991 * t996)))) + (static_cast<Real>(-1.0) * t906)) + (static_cast<Real>(-1.0) * t1133)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t1152), hk::math::abs(t45))))));
            const auto t1160 = (t1159 < static_cast<Real>(1.0));
            const auto t1161 = hk::Item<Real, 6>{t766, t847, t929, t1082, t1117, t1152};
            const auto hz0 = hk::constant<hk::extents<>>(t1160);
            const auto t1166 = (t1160 ? (t4 ? psc_t_end_i : (mut_t_i + t5)) : mut_t_i);
            mut_s[i] = hk::select(hz0, t1161, mut_s_i);
            mut_t[i] = t1166;
            mut_h[i] = (t5 * hk::math::fmin(static_cast<Real>(5.0), hk::math::fmax(static_cast<Real>(0.2), (static_cast<Real>(0.9) * (static_cast<Real>(1.0) / hk::math::sqrt(hk::math::sqrt(hk::math::sqrt(t1159))))))));
            mut_n_acc[i] = (mut_n_acc[i].get()() + (t1160 ? static_cast<Real>(1.0) : static_cast<Real>(0.0)));
            mut_n_rej[i] = (mut_n_rej[i].get()() + (t1160 ? static_cast<Real>(0.0) : static_cast<Real>(1.0)));
            if (!trm_terminated[i].eval() && (t1166 >= psc_t_end_i)) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
        }
    }
    } else {
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        if (!trm_terminated[i].eval()) {
            const auto mut_s_i = mut_s[i].get();
            const auto mut_t_i = mut_t[i].get()();
            const auto mut_h_i = mut_h[i].get()();
            const auto mut_n_acc_i = mut_n_acc[i].get()();
            const auto mut_n_rej_i = mut_n_rej[i].get()();
            const auto psc_t_end_i = psc_t_end[i].eval();
            const auto t70 = lut_fused_steps[hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(0)))].eval();
            const auto t72 = ((t70 < static_cast<Int>(0)) ? static_cast<Int>(0) : t70);
            hk::Item<Real, 6> hawk_v73_0_s = mut_s_i;
            Real hawk_v73_1_t = mut_t_i;
            Real hawk_v73_2_h = mut_h_i;
            Real hawk_v73_3_n_acc = mut_n_acc_i;
            Real hawk_v73_4_n_rej = mut_n_rej_i;
            Real hawk_v73_5_finished = static_cast<Real>(0.0);
            for (int hawk_k73_step = 0; hawk_k73_step < hawk_clamp_count(t72); ++hawk_k73_step) {
                const auto tb0 = (psc_t_end_i - hawk_v73_1_t);
                const auto tb1 = (hawk_v73_2_h >= tb0);
                const auto tb2 = (tb1 ? tb0 : hawk_v73_2_h);
                const auto tb3 = hawk_v73_0_s.eval<3>(i);
                const auto tb4 = (((hawk_v73_0_s.eval<0>(i) * hawk_v73_0_s.eval<0>(i)) + (hawk_v73_0_s.eval<1>(i) * hawk_v73_0_s.eval<1>(i))) + (hawk_v73_0_s.eval<2>(i) * hawk_v73_0_s.eval<2>(i)));
                const auto tb5 = (static_cast<Real>(1.0) / (tb4 * hk::math::sqrt(tb4)));
                const auto tb6 = (-(hawk_v73_0_s.eval<0>(i) * tb5));
                const auto tb7 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb3)));
                const auto tb8 = hawk_v73_0_s.eval<4>(i);
                const auto tb9 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb8)));
                const auto tb10 = hawk_v73_0_s.eval<5>(i);
                const auto tb11 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb10)));
                const auto tb12 = (((tb7 * tb7) + (tb9 * tb9)) + (tb11 * tb11));
                const auto tb13 = (static_cast<Real>(1.0) / (tb12 * hk::math::sqrt(tb12)));
                const auto tb14 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb6) + (static_cast<Real>(0.08333333333333333) * (-(tb7 * tb13))))));
                const auto tb15 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb3) + (static_cast<Real>(0.125) * tb14))));
                const auto tb16 = (-(hawk_v73_0_s.eval<1>(i) * tb5));
                const auto tb17 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb16) + (static_cast<Real>(0.08333333333333333) * (-(tb9 * tb13))))));
                const auto tb18 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb8) + (static_cast<Real>(0.125) * tb17))));
                const auto tb19 = (-(hawk_v73_0_s.eval<2>(i) * tb5));
                const auto tb20 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb19) + (static_cast<Real>(0.08333333333333333) * (-(tb11 * tb13))))));
                const auto tb21 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb10) + (static_cast<Real>(0.125) * tb20))));
                const auto tb22 = (((tb15 * tb15) + (tb18 * tb18)) + (tb21 * tb21));
                const auto tb23 = (static_cast<Real>(1.0) / (tb22 * hk::math::sqrt(tb22)));
                const auto tb24 = (-(tb15 * tb23));
                const auto tb25 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb3) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<3>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb6)))))));
                const auto tb26 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb8) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<4>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb16)))))));
                const auto tb27 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb10) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<5>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb19)))))));
                const auto tb28 = (((tb25 * tb25) + (tb26 * tb26)) + (tb27 * tb27));
                const auto tb29 = (static_cast<Real>(1.0) / (tb28 * hk::math::sqrt(tb28)));
                const auto tb30 = (-(tb25 * tb29));
                const auto tb31 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb6) + (static_cast<Real>(0.125) * tb30))));
                const auto tb32 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb3) + (static_cast<Real>(-1.5625) * tb14)) + (static_cast<Real>(1.5625) * tb31))));
                const auto tb33 = (-(tb26 * tb29));
                const auto tb34 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb16) + (static_cast<Real>(0.125) * tb33))));
                const auto tb35 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb8) + (static_cast<Real>(-1.5625) * tb17)) + (static_cast<Real>(1.5625) * tb34))));
                const auto tb36 = (-(tb27 * tb29));
                const auto tb37 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb19) + (static_cast<Real>(0.125) * tb36))));
                const auto tb38 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb10) + (static_cast<Real>(-1.5625) * tb20)) + (static_cast<Real>(1.5625) * tb37))));
                const auto tb39 = (((tb32 * tb32) + (tb35 * tb35)) + (tb38 * tb38));
                const auto tb40 = (static_cast<Real>(1.0) / (tb39 * hk::math::sqrt(tb39)));
                const auto tb41 = (-(tb32 * tb40));
                const auto tb42 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb6) + (static_cast<Real>(-1.5625) * tb30)) + (static_cast<Real>(1.5625) * tb24))));
                const auto tb43 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((static_cast<Real>(0.05) * tb3) + (static_cast<Real>(0.25) * tb31)) + (static_cast<Real>(0.2) * tb42))));
                const auto tb44 = (-(tb18 * tb23));
                const auto tb45 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb16) + (static_cast<Real>(-1.5625) * tb33)) + (static_cast<Real>(1.5625) * tb44))));
                const auto tb46 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((static_cast<Real>(0.05) * tb8) + (static_cast<Real>(0.25) * tb34)) + (static_cast<Real>(0.2) * tb45))));
                const auto tb47 = (-(tb21 * tb23));
                const auto tb48 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb19) + (static_cast<Real>(-1.5625) * tb36)) + (static_cast<Real>(1.5625) * tb47))));
                const auto tb49 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((static_cast<Real>(0.05) * tb10) + (static_cast<Real>(0.25) * tb37)) + (static_cast<Real>(0.2) * tb48))));
                const auto tb50 = (((tb43 * tb43) + (tb46 * tb46)) + (tb49 * tb49));
                const auto tb51 = (static_cast<Real>(1.0) / (tb50 * hk::math::sqrt(tb50)));
                const auto tb52 = (-(tb43 * tb51));
                const auto tb53 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((static_cast<Real>(0.05) * tb6) + (static_cast<Real>(0.25) * tb24)) + (static_cast<Real>(0.2) * tb41))));
                const auto tb54 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb3) + (static_cast<Real>(1.1574074074074074) * tb31)) + (static_cast<Real>(-2.4074074074074074) * tb42)) + (static_cast<Real>(2.314814814814815) * tb53))));
                const auto tb55 = (-(tb35 * tb40));
                const auto tb56 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((static_cast<Real>(0.05) * tb16) + (static_cast<Real>(0.25) * tb44)) + (static_cast<Real>(0.2) * tb55))));
                const auto tb57 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb8) + (static_cast<Real>(1.1574074074074074) * tb34)) + (static_cast<Real>(-2.4074074074074074) * tb45)) + (static_cast<Real>(2.314814814814815) * tb56))));
                const auto tb58 = (-(tb38 * tb40));
                const auto tb59 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((static_cast<Real>(0.05) * tb19) + (static_cast<Real>(0.25) * tb47)) + (static_cast<Real>(0.2) * tb58))));
                const auto tb60 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb10) + (static_cast<Real>(1.1574074074074074) * tb37)) + (static_cast<Real>(-2.4074074074074074) * tb48)) + (static_cast<Real>(2.314814814814815) * tb59))));
                const auto tb61 = (((tb54 * tb54) + (tb57 * tb57)) + (tb60 * tb60));
                const auto tb62 = (static_cast<Real>(1.0) / (tb61 * hk::math::sqrt(tb61)));
                const auto tb63 = (-(tb54 * tb62));
                const auto tb64 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb6) + (static_cast<Real>(1.1574074074074074) * tb24)) + (static_cast<Real>(-2.4074074074074074) * tb41)) + (static_cast<Real>(2.314814814814815) * tb52))));
                const auto tb65 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb3) + (static_cast<Real>(0.27111111111111114) * tb42)) + (static_cast<Real>(-0.2222222222222222) * tb53)) + (static_cast<Real>(0.014444444444444444) * tb64))));
                const auto tb66 = (-(tb46 * tb51));
                const auto tb67 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb16) + (static_cast<Real>(1.1574074074074074) * tb44)) + (static_cast<Real>(-2.4074074074074074) * tb55)) + (static_cast<Real>(2.314814814814815) * tb66))));
                const auto tb68 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb8) + (static_cast<Real>(0.27111111111111114) * tb45)) + (static_cast<Real>(-0.2222222222222222) * tb56)) + (static_cast<Real>(0.014444444444444444) * tb67))));
                const auto tb69 = (-(tb49 * tb51));
                const auto tb70 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb19) + (static_cast<Real>(1.1574074074074074) * tb47)) + (static_cast<Real>(-2.4074074074074074) * tb58)) + (static_cast<Real>(2.314814814814815) * tb69))));
                const auto tb71 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb10) + (static_cast<Real>(0.27111111111111114) * tb48)) + (static_cast<Real>(-0.2222222222222222) * tb59)) + (static_cast<Real>(0.014444444444444444) * tb70))));
                const auto tb72 = (((tb65 * tb65) + (tb68 * tb68)) + (tb71 * tb71));
                const auto tb73 = (static_cast<Real>(1.0) / (tb72 * hk::math::sqrt(tb72)));
                const auto tb74 = (-(tb65 * tb73));
                const auto tb75 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb6) + (static_cast<Real>(0.27111111111111114) * tb41)) + (static_cast<Real>(-0.2222222222222222) * tb52)) + (static_cast<Real>(0.014444444444444444) * tb63))));
                const auto tb76 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb3) + (static_cast<Real>(-8.833333333333334) * tb31)) + (static_cast<Real>(15.644444444444444) * tb42)) + (static_cast<Real>(-11.88888888888889) * tb53)) + (static_cast<Real>(0.7444444444444445) * tb64)) + (static_cast<Real>(3.0) * tb75))));
                const auto tb77 = (-(tb57 * tb62));
                const auto tb78 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb16) + (static_cast<Real>(0.27111111111111114) * tb55)) + (static_cast<Real>(-0.2222222222222222) * tb66)) + (static_cast<Real>(0.014444444444444444) * tb77))));
                const auto tb79 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb8) + (static_cast<Real>(-8.833333333333334) * tb34)) + (static_cast<Real>(15.644444444444444) * tb45)) + (static_cast<Real>(-11.88888888888889) * tb56)) + (static_cast<Real>(0.7444444444444445) * tb67)) + (static_cast<Real>(3.0) * tb78))));
                const auto tb80 = (-(tb60 * tb62));
                const auto tb81 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb19) + (static_cast<Real>(0.27111111111111114) * tb58)) + (static_cast<Real>(-0.2222222222222222) * tb69)) + (static_cast<Real>(0.014444444444444444) * tb80))));
                const auto tb82 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb10) + (static_cast<Real>(-8.833333333333334) * tb37)) + (static_cast<Real>(15.644444444444444) * tb48)) + (static_cast<Real>(-11.88888888888889) * tb59)) + (static_cast<Real>(0.7444444444444445) * tb70)) + (static_cast<Real>(3.0) * tb81))));
                const auto tb83 = (((tb76 * tb76) + (tb79 * tb79)) + (tb82 * tb82));
                const auto tb84 = (static_cast<Real>(1.0) / (tb83 * hk::math::sqrt(tb83)));
                const auto tb85 = (-(tb76 * tb84));
                const auto tb86 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb6) + (static_cast<Real>(-8.833333333333334) * tb24)) + (static_cast<Real>(15.644444444444444) * tb41)) + (static_cast<Real>(-11.88888888888889) * tb52)) + (static_cast<Real>(0.7444444444444445) * tb63)) + (static_cast<Real>(3.0) * tb74))));
                const auto tb87 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb3) + (static_cast<Real>(0.21296296296296297) * tb31)) + (static_cast<Real>(-7.229629629629629) * tb42)) + (static_cast<Real>(5.7592592592592595) * tb53)) + (static_cast<Real>(-0.31666666666666665) * tb64)) + (static_cast<Real>(2.8333333333333335) * tb75)) + (static_cast<Real>(-0.08333333333333333) * tb86))));
                const auto tb88 = (-(tb68 * tb73));
                const auto tb89 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb16) + (static_cast<Real>(-8.833333333333334) * tb44)) + (static_cast<Real>(15.644444444444444) * tb55)) + (static_cast<Real>(-11.88888888888889) * tb66)) + (static_cast<Real>(0.7444444444444445) * tb77)) + (static_cast<Real>(3.0) * tb88))));
                const auto tb90 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb8) + (static_cast<Real>(0.21296296296296297) * tb34)) + (static_cast<Real>(-7.229629629629629) * tb45)) + (static_cast<Real>(5.7592592592592595) * tb56)) + (static_cast<Real>(-0.31666666666666665) * tb67)) + (static_cast<Real>(2.8333333333333335) * tb78)) + (static_cast<Real>(-0.08333333333333333) * tb89))));
                const auto tb91 = (-(tb71 * tb73));
                const auto tb92 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb19) + (static_cast<Real>(-8.833333333333334) * tb47)) + (static_cast<Real>(15.644444444444444) * tb58)) + (static_cast<Real>(-11.88888888888889) * tb69)) + (static_cast<Real>(0.7444444444444445) * tb80)) + (static_cast<Real>(3.0) * tb91))));
                const auto tb93 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb10) + (static_cast<Real>(0.21296296296296297) * tb37)) + (static_cast<Real>(-7.229629629629629) * tb48)) + (static_cast<Real>(5.7592592592592595) * tb59)) + (static_cast<Real>(-0.31666666666666665) * tb70)) + (static_cast<Real>(2.8333333333333335) * tb81)) + (static_cast<Real>(-0.08333333333333333) * tb92))));
                const auto tb94 = (((tb87 * tb87) + (tb90 * tb90)) + (tb93 * tb93));
                const auto tb95 = (static_cast<Real>(1.0) / (tb94 * hk::math::sqrt(tb94)));
                const auto tb96 = (-(tb87 * tb95));
                const auto tb97 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb6) + (static_cast<Real>(-0.14634146341463414) * tb52)) + (static_cast<Real>(-0.014634146341463415) * tb63)) + (static_cast<Real>(-0.07317073170731707) * tb74)) + (static_cast<Real>(0.07317073170731707) * tb85)) + (static_cast<Real>(0.14634146341463414) * tb96))));
                const auto tb98 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb6) + (static_cast<Real>(0.21296296296296297) * tb24)) + (static_cast<Real>(-7.229629629629629) * tb41)) + (static_cast<Real>(5.7592592592592595) * tb52)) + (static_cast<Real>(-0.31666666666666665) * tb63)) + (static_cast<Real>(2.8333333333333335) * tb74)) + (static_cast<Real>(-0.08333333333333333) * tb85))));
                const auto tb99 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb3) + (static_cast<Real>(-0.14634146341463414) * tb53)) + (static_cast<Real>(-0.014634146341463415) * tb64)) + (static_cast<Real>(-0.07317073170731707) * tb75)) + (static_cast<Real>(0.07317073170731707) * tb86)) + (static_cast<Real>(0.14634146341463414) * tb98))));
                const auto tb100 = (-(tb79 * tb84));
                const auto tb101 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb16) + (static_cast<Real>(0.21296296296296297) * tb44)) + (static_cast<Real>(-7.229629629629629) * tb55)) + (static_cast<Real>(5.7592592592592595) * tb66)) + (static_cast<Real>(-0.31666666666666665) * tb77)) + (static_cast<Real>(2.8333333333333335) * tb88)) + (static_cast<Real>(-0.08333333333333333) * tb100))));
                const auto tb102 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb8) + (static_cast<Real>(-0.14634146341463414) * tb56)) + (static_cast<Real>(-0.014634146341463415) * tb67)) + (static_cast<Real>(-0.07317073170731707) * tb78)) + (static_cast<Real>(0.07317073170731707) * tb89)) + (static_cast<Real>(0.14634146341463414) * tb101))));
                const auto tb103 = (-(tb82 * tb84));
                const auto tb104 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb19) + (static_cast<Real>(0.21296296296296297) * tb47)) + (static_cast<Real>(-7.229629629629629) * tb58)) + (static_cast<Real>(5.7592592592592595) * tb69)) + (static_cast<Real>(-0.31666666666666665) * tb80)) + (static_cast<Real>(2.8333333333333335) * tb91)) + (static_cast<Real>(-0.08333333333333333) * tb103))));
                const auto tb105 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb10) + (static_cast<Real>(-0.14634146341463414) * tb59)) + (static_cast<Real>(-0.014634146341463415) * tb70)) + (static_cast<Real>(-0.07317073170731707) * tb81)) + (static_cast<Real>(0.07317073170731707) * tb92)) + (static_cast<Real>(0.14634146341463414) * tb104))));
                const auto tb106 = (((tb99 * tb99) + (tb102 * tb102)) + (tb105 * tb105));
                const auto tb107 = (static_cast<Real>(1.0) / (tb106 * hk::math::sqrt(tb106)));
                const auto tb108 = (-(tb99 * tb107));
                const auto tb109 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb6) + (static_cast<Real>(-2.0792682926829267) * tb24)) + (static_cast<Real>(4.3863414634146345) * tb41)) + (static_cast<Real>(-3.524390243902439) * tb52)) + (static_cast<Real>(0.5348780487804878) * tb63)) + (static_cast<Real>(0.6219512195121951) * tb74)) + (static_cast<Real>(0.20121951219512196) * tb85)) + (static_cast<Real>(0.2926829268292683) * tb96)) + (static_cast<Real>(1.0) * tb108))));
                const auto tb110 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb53) + (static_cast<Real>(0.2571428571428571) * tb64)) + (static_cast<Real>(0.2571428571428571) * tb75)) + (static_cast<Real>(0.03214285714285714) * tb86)) + (static_cast<Real>(0.03214285714285714) * tb98)) + (static_cast<Real>(0.04880952380952381) * tb97)) + (static_cast<Real>(0.04880952380952381) * tb109))));
                const auto tb111 = (-(tb90 * tb95));
                const auto tb112 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb16) + (static_cast<Real>(-0.14634146341463414) * tb66)) + (static_cast<Real>(-0.014634146341463415) * tb77)) + (static_cast<Real>(-0.07317073170731707) * tb88)) + (static_cast<Real>(0.07317073170731707) * tb100)) + (static_cast<Real>(0.14634146341463414) * tb111))));
                const auto tb113 = (-(tb102 * tb107));
                const auto tb114 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb16) + (static_cast<Real>(-2.0792682926829267) * tb44)) + (static_cast<Real>(4.3863414634146345) * tb55)) + (static_cast<Real>(-3.524390243902439) * tb66)) + (static_cast<Real>(0.5348780487804878) * tb77)) + (static_cast<Real>(0.6219512195121951) * tb88)) + (static_cast<Real>(0.20121951219512196) * tb100)) + (static_cast<Real>(0.2926829268292683) * tb111)) + (static_cast<Real>(1.0) * tb113))));
                const auto tb115 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb56) + (static_cast<Real>(0.2571428571428571) * tb67)) + (static_cast<Real>(0.2571428571428571) * tb78)) + (static_cast<Real>(0.03214285714285714) * tb89)) + (static_cast<Real>(0.03214285714285714) * tb101)) + (static_cast<Real>(0.04880952380952381) * tb112)) + (static_cast<Real>(0.04880952380952381) * tb114))));
                const auto tb116 = (-(tb93 * tb95));
                const auto tb117 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb19) + (static_cast<Real>(-0.14634146341463414) * tb69)) + (static_cast<Real>(-0.014634146341463415) * tb80)) + (static_cast<Real>(-0.07317073170731707) * tb91)) + (static_cast<Real>(0.07317073170731707) * tb103)) + (static_cast<Real>(0.14634146341463414) * tb116))));
                const auto tb118 = (-(tb105 * tb107));
                const auto tb119 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb19) + (static_cast<Real>(-2.0792682926829267) * tb47)) + (static_cast<Real>(4.3863414634146345) * tb58)) + (static_cast<Real>(-3.524390243902439) * tb69)) + (static_cast<Real>(0.5348780487804878) * tb80)) + (static_cast<Real>(0.6219512195121951) * tb91)) + (static_cast<Real>(0.20121951219512196) * tb103)) + (static_cast<Real>(0.2926829268292683) * tb116)) + (static_cast<Real>(1.0) * tb118))));
                const auto tb120 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb59) + (static_cast<Real>(0.2571428571428571) * tb70)) + (static_cast<Real>(0.2571428571428571) * tb81)) + (static_cast<Real>(0.03214285714285714) * tb92)) + (static_cast<Real>(0.03214285714285714) * tb104)) + (static_cast<Real>(0.04880952380952381) * tb117)) + (static_cast<Real>(0.04880952380952381) * tb119))));
                const auto tb121 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb3) + (static_cast<Real>(-2.0792682926829267) * tb31)) + (static_cast<Real>(4.3863414634146345) * tb42)) + (static_cast<Real>(-3.6707317073170733) * tb53)) + (static_cast<Real>(0.5202439024390244) * tb64)) + (static_cast<Real>(0.5487804878048781) * tb75)) + (static_cast<Real>(0.27439024390243905) * tb86)) + (static_cast<Real>(0.43902439024390244) * tb98))));
                const auto tb122 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb8) + (static_cast<Real>(-2.0792682926829267) * tb34)) + (static_cast<Real>(4.3863414634146345) * tb45)) + (static_cast<Real>(-3.6707317073170733) * tb56)) + (static_cast<Real>(0.5202439024390244) * tb67)) + (static_cast<Real>(0.5487804878048781) * tb78)) + (static_cast<Real>(0.27439024390243905) * tb89)) + (static_cast<Real>(0.43902439024390244) * tb101))));
                const auto tb123 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb10) + (static_cast<Real>(-2.0792682926829267) * tb37)) + (static_cast<Real>(4.3863414634146345) * tb48)) + (static_cast<Real>(-3.6707317073170733) * tb59)) + (static_cast<Real>(0.5202439024390244) * tb70)) + (static_cast<Real>(0.5487804878048781) * tb81)) + (static_cast<Real>(0.27439024390243905) * tb92)) + (static_cast<Real>(0.43902439024390244) * tb104))));
                const auto tb124 = (((tb121 * tb121) + (tb122 * tb122)) + (tb123 * tb123));
                const auto tb125 = (static_cast<Real>(1.0) / (tb124 * hk::math::sqrt(tb124)));
                const auto tb126 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb3) + (static_cast<Real>(-2.0792682926829267) * tb31)) + (static_cast<Real>(4.3863414634146345) * tb42)) + (static_cast<Real>(-3.524390243902439) * tb53)) + (static_cast<Real>(0.5348780487804878) * tb64)) + (static_cast<Real>(0.6219512195121951) * tb75)) + (static_cast<Real>(0.20121951219512196) * tb86)) + (static_cast<Real>(0.2926829268292683) * tb98)) + (static_cast<Real>(1.0) * tb97))));
                const auto tb127 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb8) + (static_cast<Real>(-2.0792682926829267) * tb34)) + (static_cast<Real>(4.3863414634146345) * tb45)) + (static_cast<Real>(-3.524390243902439) * tb56)) + (static_cast<Real>(0.5348780487804878) * tb67)) + (static_cast<Real>(0.6219512195121951) * tb78)) + (static_cast<Real>(0.20121951219512196) * tb89)) + (static_cast<Real>(0.2926829268292683) * tb101)) + (static_cast<Real>(1.0) * tb112))));
                const auto tb128 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb10) + (static_cast<Real>(-2.0792682926829267) * tb37)) + (static_cast<Real>(4.3863414634146345) * tb48)) + (static_cast<Real>(-3.524390243902439) * tb59)) + (static_cast<Real>(0.5348780487804878) * tb70)) + (static_cast<Real>(0.6219512195121951) * tb81)) + (static_cast<Real>(0.20121951219512196) * tb92)) + (static_cast<Real>(0.2926829268292683) * tb104)) + (static_cast<Real>(1.0) * tb117))));
                const auto tb129 = (((tb126 * tb126) + (tb127 * tb127)) + (tb128 * tb128));
                const auto tb130 = (static_cast<Real>(1.0) / (tb129 * hk::math::sqrt(tb129)));
                const auto tb131 = (-(tb126 * tb130));
                const auto tb132 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb52) + (static_cast<Real>(0.2571428571428571) * tb63)) + (static_cast<Real>(0.2571428571428571) * tb74)) + (static_cast<Real>(0.03214285714285714) * tb85)) + (static_cast<Real>(0.03214285714285714) * tb96)) + (static_cast<Real>(0.04880952380952381) * tb108)) + (static_cast<Real>(0.04880952380952381) * tb131))));
                const auto tb133 = (-(tb127 * tb130));
                const auto tb134 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb66) + (static_cast<Real>(0.2571428571428571) * tb77)) + (static_cast<Real>(0.2571428571428571) * tb88)) + (static_cast<Real>(0.03214285714285714) * tb100)) + (static_cast<Real>(0.03214285714285714) * tb111)) + (static_cast<Real>(0.04880952380952381) * tb113)) + (static_cast<Real>(0.04880952380952381) * tb133))));
                const auto tb135 = (-(tb128 * tb130));
                const auto tb136 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb69) + (static_cast<Real>(0.2571428571428571) * tb80)) + (static_cast<Real>(0.2571428571428571) * tb91)) + (static_cast<Real>(0.03214285714285714) * tb103)) + (static_cast<Real>(0.03214285714285714) * tb116)) + (static_cast<Real>(0.04880952380952381) * tb118)) + (static_cast<Real>(0.04880952380952381) * tb135))));
                const auto tb137 = hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax((hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb3) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb6) + (static_cast<Real>(-2.0792682926829267) * tb24)) + (static_cast<Real>(4.3863414634146345) * tb41)) + (static_cast<Real>(-3.6707317073170733) * tb52)) + (static_cast<Real>(0.5202439024390244) * tb63)) + (static_cast<Real>(0.5487804878048781) * tb74)) + (static_cast<Real>(0.27439024390243905) * tb85)) + (static_cast<Real>(0.43902439024390244) * tb96)))))) + (static_cast<Real>(-1.0) * tb97)) + (static_cast<Real>(-1.0) * tb109)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb110), hk::math::abs(hawk_v73_0_s.eval<0>(i)))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb8) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb16) + (static_cast<Real>(-2.0792682926829267) * tb44)) + (static_cast<Real>(4.3863414634146345) * tb55)) + (static_cast<Real>(-3.6707317073170733) * tb66)) + (static_cast<Real>(0.5202439024390244) * tb77)) + (static_cast<Real>(0.5487804878048781) * tb88)) + (static_cast<Real>(0.27439024390243905) * tb100)) + (static_cast<Real>(0.43902439024390244) * tb111)))))) + (static_cast<Real>(-1.0) * tb112)) + (static_cast<Real>(-1.0) * tb114)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb115), hk::math::abs(hawk_v73_0_s.eval<1>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb10) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb19) + (static_cast<Real>(-2.0792682926829267) * tb47)) + (static_cast<Real>(4.3863414634146345) * tb58)) + (static_cast<Real>(-3.6707317073170733) * tb69)) + (static_cast<Real>(0.5202439024390244) * tb80)) + (static_cast<Real>(0.5487804878048781) * tb91)) + (static_cast<Real>(0.27439024390243905) * tb103)) + (static_cast<Real>(0.43902439024390244) * tb116)))))) + (static_cast<Real>(-1.0) * tb117)) + (static_cast<Real>(-1.0) * tb119)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb120), hk::math::abs(hawk_v73_0_s.eval<2>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb6) + (static_cast<Real>(1.0) * (-(tb121 * tb125)))) + (static_cast<Real>(-1.0) * tb108)) + (static_cast<Real>(-1.0) * tb131)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb132), hk::math::abs(hawk_v73_0_s.eval<3>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb16) + (static_cast<Real>(1.0) * (-(tb122 * tb125)))) + (static_cast<Real>(-1.0) * tb113)) + (static_cast<Real>(-1.0) * tb133)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb134), hk::math::abs(hawk_v73_0_s.eval<4>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb19) + (static_cast<Real>(1.0) * (-(tb123 * tb125)))) + (static_cast<Real>(-1.0) * tb118)) + (static_cast<Real>(-1.0) * tb135)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb136), hk::math::abs(hawk_v73_0_s.eval<5>(i)))))));
                const auto tb138 = (tb137 < static_cast<Real>(1.0));
                const auto tb139 = hk::Item<Real, 6>{tb110, tb115, tb120, tb132, tb134, tb136};
                const auto hz0 = hk::constant<hk::extents<>>(tb138);
                const auto tb140 = (tb1 ? psc_t_end_i : (hawk_v73_1_t + tb2));
                const auto tb141 = (tb138 ? tb140 : hawk_v73_1_t);
                const auto tb142 = hk::math::fmin(static_cast<Real>(5.0), hk::math::fmax(static_cast<Real>(0.2), (static_cast<Real>(0.9) * (static_cast<Real>(1.0) / hk::math::sqrt(hk::math::sqrt(hk::math::sqrt(tb137)))))));
                const auto tb143 = (tb138 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                const auto tb144 = (tb138 ? static_cast<Real>(0.0) : static_cast<Real>(1.0));
                const auto tb145 = (tb141 >= psc_t_end_i);
                const hk::Item<Real, 6> hawk_n73_0 = hk::select(hz0, tb139, hawk_v73_0_s);
                const Real hawk_n73_1 = tb141;
                const Real hawk_n73_2 = (tb2 * tb142);
                const Real hawk_n73_3 = (hawk_v73_3_n_acc + tb143);
                const Real hawk_n73_4 = (hawk_v73_4_n_rej + tb144);
                const Real hawk_n73_5 = (tb145 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                const bool hawk_x73 = tb145;
                hawk_v73_0_s = hawk_n73_0;
                hawk_v73_1_t = hawk_n73_1;
                hawk_v73_2_h = hawk_n73_2;
                hawk_v73_3_n_acc = hawk_n73_3;
                hawk_v73_4_n_rej = hawk_n73_4;
                hawk_v73_5_finished = hawk_n73_5;
                if (hawk_x73) break;
            }
            mut_s[i] = hawk_v73_0_s;
            mut_t[i] = hawk_v73_1_t;
            mut_h[i] = hawk_v73_2_h;
            mut_n_acc[i] = hawk_v73_3_n_acc;
            mut_n_rej[i] = hawk_v73_4_n_rej;
            if (!trm_terminated[i].eval() && (hawk_v73_5_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
        }
    }
    }
}

extern "C" __global__ void __launch_bounds__(256) orbit_persist(
    hk::abi::ScalarHandle p_mut_h,
    hk::abi::ScalarHandle p_mut_n_acc,
    hk::abi::ScalarHandle p_mut_n_rej,
    hk::abi::GRefMirror p_mut_s,
    hk::abi::ScalarHandle p_mut_t,
    hk::abi::ScalarHandle p_psc_t_end,
    hk::abi::ScalarHandle p_lut_finished_count,
    hk::abi::ScalarHandle p_lut_fused_steps,
    hk::abi::ScalarHandle p_trm_terminated,
    long long base,
    long long count,
    long long nSamples,
    unsigned int* hawk_next,
    unsigned long long* hawk_util,
    unsigned int* hawk_steps,
    unsigned long long* hawk_stepsum,
    unsigned int hawk_chunk)
{
    const hk::ScalarOut<Real> mut_h(p_mut_h);
    (void)mut_h;
    const hk::ScalarOut<Real> mut_n_acc(p_mut_n_acc);
    (void)mut_n_acc;
    const hk::ScalarOut<Real> mut_n_rej(p_mut_n_rej);
    (void)mut_n_rej;
    const hk::VecOut<Real, 6> mut_s(p_mut_s);
    (void)mut_s;
    const hk::ScalarOut<Real> mut_t(p_mut_t);
    (void)mut_t;
    const hk::ScalarIn<Real> psc_t_end(p_psc_t_end);
    (void)psc_t_end;
    const hk::ScalarIn<std::uint32_t> lut_finished_count(p_lut_finished_count);
    (void)lut_finished_count;
    const hk::ScalarIn<Int> lut_fused_steps(p_lut_fused_steps);
    (void)lut_fused_steps;
    const hk::MaskView trm_terminated(p_trm_terminated);
    (void)trm_terminated;
    const hk::MaskView trm_terminated_w(p_trm_terminated);
    (void)trm_terminated_w;
    hk::Item<Real, 6> hk_c0{};
    Real hk_c1{};
    Real hk_c2{};
    Real hk_c3{};
    Real hk_c4{};
    Real hk_c5{};
    Real hk_l0{};
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
                            const auto mut_s_i = mut_s[i].get();
                            const auto mut_t_i = mut_t[i].get()();
                            const auto mut_h_i = mut_h[i].get()();
                            const auto mut_n_acc_i = mut_n_acc[i].get()();
                            const auto mut_n_rej_i = mut_n_rej[i].get()();
                            const auto psc_t_end_i = psc_t_end[i].eval();
                            const auto t70 = lut_fused_steps[hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(0)))].eval();
                            const auto t72 = ((t70 < static_cast<Int>(0)) ? static_cast<Int>(0) : t70);
                        hk_c0 = mut_s_i;
                        hk_c1 = mut_t_i;
                        hk_c2 = mut_h_i;
                        hk_c3 = mut_n_acc_i;
                        hk_c4 = mut_n_rej_i;
                        hk_c5 = static_cast<Real>(0.0);
                        hk_l0 = psc_t_end_i;
                        hk_budget = static_cast<unsigned>(hawk_clamp_count(t72));
                        hk_trip = 0u;
                        hk_has = true;
                        if (hk_budget == 0u) {
                            const hk::Item<Real, 6> hawk_v73_0_s = hk_c0;
                            const Real hawk_v73_1_t = hk_c1;
                            const Real hawk_v73_2_h = hk_c2;
                            const Real hawk_v73_3_n_acc = hk_c3;
                            const Real hawk_v73_4_n_rej = hk_c4;
                            const Real hawk_v73_5_finished = hk_c5;
                            (void)hawk_v73_0_s;
                            (void)hawk_v73_1_t;
                            (void)hawk_v73_2_h;
                            (void)hawk_v73_3_n_acc;
                            (void)hawk_v73_4_n_rej;
                            (void)hawk_v73_5_finished;
                                mut_s[i] = hawk_v73_0_s;
                            mut_t[i] = hawk_v73_1_t;
                            mut_h[i] = hawk_v73_2_h;
                            mut_n_acc[i] = hawk_v73_3_n_acc;
                            mut_n_rej[i] = hawk_v73_4_n_rej;
                            if (!trm_terminated[i].eval() && (hawk_v73_5_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; ++hk_fin; }
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
                const int hawk_k73_step = static_cast<int>(hk_trip);
                (void)hawk_k73_step;
                const hk::Item<Real, 6> hawk_v73_0_s = hk_c0;
                const Real hawk_v73_1_t = hk_c1;
                const Real hawk_v73_2_h = hk_c2;
                const Real hawk_v73_3_n_acc = hk_c3;
                const Real hawk_v73_4_n_rej = hk_c4;
                const Real hawk_v73_5_finished = hk_c5;
                const Real psc_t_end_i = hk_l0;
                (void)psc_t_end_i;
                                const auto tb0 = (psc_t_end_i - hawk_v73_1_t);
                                const auto tb1 = (hawk_v73_2_h >= tb0);
                                const auto tb2 = (tb1 ? tb0 : hawk_v73_2_h);
                                const auto tb3 = hawk_v73_0_s.eval<3>(i);
                                const auto tb4 = (((hawk_v73_0_s.eval<0>(i) * hawk_v73_0_s.eval<0>(i)) + (hawk_v73_0_s.eval<1>(i) * hawk_v73_0_s.eval<1>(i))) + (hawk_v73_0_s.eval<2>(i) * hawk_v73_0_s.eval<2>(i)));
                                const auto tb5 = (static_cast<Real>(1.0) / (tb4 * hk::math::sqrt(tb4)));
                                const auto tb6 = (-(hawk_v73_0_s.eval<0>(i) * tb5));
                                const auto tb7 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb3)));
                                const auto tb8 = hawk_v73_0_s.eval<4>(i);
                                const auto tb9 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb8)));
                                const auto tb10 = hawk_v73_0_s.eval<5>(i);
                                const auto tb11 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb10)));
                                const auto tb12 = (((tb7 * tb7) + (tb9 * tb9)) + (tb11 * tb11));
                                const auto tb13 = (static_cast<Real>(1.0) / (tb12 * hk::math::sqrt(tb12)));
                                const auto tb14 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb6) + (static_cast<Real>(0.08333333333333333) * (-(tb7 * tb13))))));
                                const auto tb15 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb3) + (static_cast<Real>(0.125) * tb14))));
                                const auto tb16 = (-(hawk_v73_0_s.eval<1>(i) * tb5));
                                const auto tb17 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb16) + (static_cast<Real>(0.08333333333333333) * (-(tb9 * tb13))))));
                                const auto tb18 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb8) + (static_cast<Real>(0.125) * tb17))));
                                const auto tb19 = (-(hawk_v73_0_s.eval<2>(i) * tb5));
                                const auto tb20 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb19) + (static_cast<Real>(0.08333333333333333) * (-(tb11 * tb13))))));
                                const auto tb21 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb10) + (static_cast<Real>(0.125) * tb20))));
                                const auto tb22 = (((tb15 * tb15) + (tb18 * tb18)) + (tb21 * tb21));
                                const auto tb23 = (static_cast<Real>(1.0) / (tb22 * hk::math::sqrt(tb22)));
                                const auto tb24 = (-(tb15 * tb23));
                                const auto tb25 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb3) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<3>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb6)))))));
                                const auto tb26 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb8) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<4>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb16)))))));
                                const auto tb27 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb10) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<5>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb19)))))));
                                const auto tb28 = (((tb25 * tb25) + (tb26 * tb26)) + (tb27 * tb27));
                                const auto tb29 = (static_cast<Real>(1.0) / (tb28 * hk::math::sqrt(tb28)));
                                const auto tb30 = (-(tb25 * tb29));
                                const auto tb31 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb6) + (static_cast<Real>(0.125) * tb30))));
                                const auto tb32 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb3) + (static_cast<Real>(-1.5625) * tb14)) + (static_cast<Real>(1.5625) * tb31))));
                                const auto tb33 = (-(tb26 * tb29));
                                const auto tb34 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb16) + (static_cast<Real>(0.125) * tb33))));
                                const auto tb35 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb8) + (static_cast<Real>(-1.5625) * tb17)) + (static_cast<Real>(1.5625) * tb34))));
                                const auto tb36 = (-(tb27 * tb29));
                                const auto tb37 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb19) + (static_cast<Real>(0.125) * tb36))));
                                const auto tb38 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb10) + (static_cast<Real>(-1.5625) * tb20)) + (static_cast<Real>(1.5625) * tb37))));
                                const auto tb39 = (((tb32 * tb32) + (tb35 * tb35)) + (tb38 * tb38));
                                const auto tb40 = (static_cast<Real>(1.0) / (tb39 * hk::math::sqrt(tb39)));
                                const auto tb41 = (-(tb32 * tb40));
                                const auto tb42 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb6) + (static_cast<Real>(-1.5625) * tb30)) + (static_cast<Real>(1.5625) * tb24))));
                                const auto tb43 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((static_cast<Real>(0.05) * tb3) + (static_cast<Real>(0.25) * tb31)) + (static_cast<Real>(0.2) * tb42))));
                                const auto tb44 = (-(tb18 * tb23));
                                const auto tb45 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb16) + (static_cast<Real>(-1.5625) * tb33)) + (static_cast<Real>(1.5625) * tb44))));
                                const auto tb46 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((static_cast<Real>(0.05) * tb8) + (static_cast<Real>(0.25) * tb34)) + (static_cast<Real>(0.2) * tb45))));
                                const auto tb47 = (-(tb21 * tb23));
                                const auto tb48 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb19) + (static_cast<Real>(-1.5625) * tb36)) + (static_cast<Real>(1.5625) * tb47))));
                                const auto tb49 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((static_cast<Real>(0.05) * tb10) + (static_cast<Real>(0.25) * tb37)) + (static_cast<Real>(0.2) * tb48))));
                                const auto tb50 = (((tb43 * tb43) + (tb46 * tb46)) + (tb49 * tb49));
                                const auto tb51 = (static_cast<Real>(1.0) / (tb50 * hk::math::sqrt(tb50)));
                                const auto tb52 = (-(tb43 * tb51));
                                const auto tb53 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((static_cast<Real>(0.05) * tb6) + (static_cast<Real>(0.25) * tb24)) + (static_cast<Real>(0.2) * tb41))));
                                const auto tb54 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb3) + (static_cast<Real>(1.1574074074074074) * tb31)) + (static_cast<Real>(-2.4074074074074074) * tb42)) + (static_cast<Real>(2.314814814814815) * tb53))));
                                const auto tb55 = (-(tb35 * tb40));
                                const auto tb56 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((static_cast<Real>(0.05) * tb16) + (static_cast<Real>(0.25) * tb44)) + (static_cast<Real>(0.2) * tb55))));
                                const auto tb57 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb8) + (static_cast<Real>(1.1574074074074074) * tb34)) + (static_cast<Real>(-2.4074074074074074) * tb45)) + (static_cast<Real>(2.314814814814815) * tb56))));
                                const auto tb58 = (-(tb38 * tb40));
                                const auto tb59 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((static_cast<Real>(0.05) * tb19) + (static_cast<Real>(0.25) * tb47)) + (static_cast<Real>(0.2) * tb58))));
                                const auto tb60 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb10) + (static_cast<Real>(1.1574074074074074) * tb37)) + (static_cast<Real>(-2.4074074074074074) * tb48)) + (static_cast<Real>(2.314814814814815) * tb59))));
                                const auto tb61 = (((tb54 * tb54) + (tb57 * tb57)) + (tb60 * tb60));
                                const auto tb62 = (static_cast<Real>(1.0) / (tb61 * hk::math::sqrt(tb61)));
                                const auto tb63 = (-(tb54 * tb62));
                                const auto tb64 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb6) + (static_cast<Real>(1.1574074074074074) * tb24)) + (static_cast<Real>(-2.4074074074074074) * tb41)) + (static_cast<Real>(2.314814814814815) * tb52))));
                                const auto tb65 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb3) + (static_cast<Real>(0.27111111111111114) * tb42)) + (static_cast<Real>(-0.2222222222222222) * tb53)) + (static_cast<Real>(0.014444444444444444) * tb64))));
                                const auto tb66 = (-(tb46 * tb51));
                                const auto tb67 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb16) + (static_cast<Real>(1.1574074074074074) * tb44)) + (static_cast<Real>(-2.4074074074074074) * tb55)) + (static_cast<Real>(2.314814814814815) * tb66))));
                                const auto tb68 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb8) + (static_cast<Real>(0.27111111111111114) * tb45)) + (static_cast<Real>(-0.2222222222222222) * tb56)) + (static_cast<Real>(0.014444444444444444) * tb67))));
                                const auto tb69 = (-(tb49 * tb51));
                                const auto tb70 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb19) + (static_cast<Real>(1.1574074074074074) * tb47)) + (static_cast<Real>(-2.4074074074074074) * tb58)) + (static_cast<Real>(2.314814814814815) * tb69))));
                                const auto tb71 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb10) + (static_cast<Real>(0.27111111111111114) * tb48)) + (static_cast<Real>(-0.2222222222222222) * tb59)) + (static_cast<Real>(0.014444444444444444) * tb70))));
                                const auto tb72 = (((tb65 * tb65) + (tb68 * tb68)) + (tb71 * tb71));
                                const auto tb73 = (static_cast<Real>(1.0) / (tb72 * hk::math::sqrt(tb72)));
                                const auto tb74 = (-(tb65 * tb73));
                                const auto tb75 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb6) + (static_cast<Real>(0.27111111111111114) * tb41)) + (static_cast<Real>(-0.2222222222222222) * tb52)) + (static_cast<Real>(0.014444444444444444) * tb63))));
                                const auto tb76 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb3) + (static_cast<Real>(-8.833333333333334) * tb31)) + (static_cast<Real>(15.644444444444444) * tb42)) + (static_cast<Real>(-11.88888888888889) * tb53)) + (static_cast<Real>(0.7444444444444445) * tb64)) + (static_cast<Real>(3.0) * tb75))));
                                const auto tb77 = (-(tb57 * tb62));
                                const auto tb78 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb16) + (static_cast<Real>(0.27111111111111114) * tb55)) + (static_cast<Real>(-0.2222222222222222) * tb66)) + (static_cast<Real>(0.014444444444444444) * tb77))));
                                const auto tb79 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb8) + (static_cast<Real>(-8.833333333333334) * tb34)) + (static_cast<Real>(15.644444444444444) * tb45)) + (static_cast<Real>(-11.88888888888889) * tb56)) + (static_cast<Real>(0.7444444444444445) * tb67)) + (static_cast<Real>(3.0) * tb78))));
                                const auto tb80 = (-(tb60 * tb62));
                                const auto tb81 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb19) + (static_cast<Real>(0.27111111111111114) * tb58)) + (static_cast<Real>(-0.2222222222222222) * tb69)) + (static_cast<Real>(0.014444444444444444) * tb80))));
                                const auto tb82 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb10) + (static_cast<Real>(-8.833333333333334) * tb37)) + (static_cast<Real>(15.644444444444444) * tb48)) + (static_cast<Real>(-11.88888888888889) * tb59)) + (static_cast<Real>(0.7444444444444445) * tb70)) + (static_cast<Real>(3.0) * tb81))));
                                const auto tb83 = (((tb76 * tb76) + (tb79 * tb79)) + (tb82 * tb82));
                                const auto tb84 = (static_cast<Real>(1.0) / (tb83 * hk::math::sqrt(tb83)));
                                const auto tb85 = (-(tb76 * tb84));
                                const auto tb86 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb6) + (static_cast<Real>(-8.833333333333334) * tb24)) + (static_cast<Real>(15.644444444444444) * tb41)) + (static_cast<Real>(-11.88888888888889) * tb52)) + (static_cast<Real>(0.7444444444444445) * tb63)) + (static_cast<Real>(3.0) * tb74))));
                                const auto tb87 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb3) + (static_cast<Real>(0.21296296296296297) * tb31)) + (static_cast<Real>(-7.229629629629629) * tb42)) + (static_cast<Real>(5.7592592592592595) * tb53)) + (static_cast<Real>(-0.31666666666666665) * tb64)) + (static_cast<Real>(2.8333333333333335) * tb75)) + (static_cast<Real>(-0.08333333333333333) * tb86))));
                                const auto tb88 = (-(tb68 * tb73));
                                const auto tb89 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb16) + (static_cast<Real>(-8.833333333333334) * tb44)) + (static_cast<Real>(15.644444444444444) * tb55)) + (static_cast<Real>(-11.88888888888889) * tb66)) + (static_cast<Real>(0.7444444444444445) * tb77)) + (static_cast<Real>(3.0) * tb88))));
                                const auto tb90 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb8) + (static_cast<Real>(0.21296296296296297) * tb34)) + (static_cast<Real>(-7.229629629629629) * tb45)) + (static_cast<Real>(5.7592592592592595) * tb56)) + (static_cast<Real>(-0.31666666666666665) * tb67)) + (static_cast<Real>(2.8333333333333335) * tb78)) + (static_cast<Real>(-0.08333333333333333) * tb89))));
                                const auto tb91 = (-(tb71 * tb73));
                                const auto tb92 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb19) + (static_cast<Real>(-8.833333333333334) * tb47)) + (static_cast<Real>(15.644444444444444) * tb58)) + (static_cast<Real>(-11.88888888888889) * tb69)) + (static_cast<Real>(0.7444444444444445) * tb80)) + (static_cast<Real>(3.0) * tb91))));
                                const auto tb93 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb10) + (static_cast<Real>(0.21296296296296297) * tb37)) + (static_cast<Real>(-7.229629629629629) * tb48)) + (static_cast<Real>(5.7592592592592595) * tb59)) + (static_cast<Real>(-0.31666666666666665) * tb70)) + (static_cast<Real>(2.8333333333333335) * tb81)) + (static_cast<Real>(-0.08333333333333333) * tb92))));
                                const auto tb94 = (((tb87 * tb87) + (tb90 * tb90)) + (tb93 * tb93));
                                const auto tb95 = (static_cast<Real>(1.0) / (tb94 * hk::math::sqrt(tb94)));
                                const auto tb96 = (-(tb87 * tb95));
                                const auto tb97 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb6) + (static_cast<Real>(-0.14634146341463414) * tb52)) + (static_cast<Real>(-0.014634146341463415) * tb63)) + (static_cast<Real>(-0.07317073170731707) * tb74)) + (static_cast<Real>(0.07317073170731707) * tb85)) + (static_cast<Real>(0.14634146341463414) * tb96))));
                                const auto tb98 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb6) + (static_cast<Real>(0.21296296296296297) * tb24)) + (static_cast<Real>(-7.229629629629629) * tb41)) + (static_cast<Real>(5.7592592592592595) * tb52)) + (static_cast<Real>(-0.31666666666666665) * tb63)) + (static_cast<Real>(2.8333333333333335) * tb74)) + (static_cast<Real>(-0.08333333333333333) * tb85))));
                                const auto tb99 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb3) + (static_cast<Real>(-0.14634146341463414) * tb53)) + (static_cast<Real>(-0.014634146341463415) * tb64)) + (static_cast<Real>(-0.07317073170731707) * tb75)) + (static_cast<Real>(0.07317073170731707) * tb86)) + (static_cast<Real>(0.14634146341463414) * tb98))));
                                const auto tb100 = (-(tb79 * tb84));
                                const auto tb101 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb16) + (static_cast<Real>(0.21296296296296297) * tb44)) + (static_cast<Real>(-7.229629629629629) * tb55)) + (static_cast<Real>(5.7592592592592595) * tb66)) + (static_cast<Real>(-0.31666666666666665) * tb77)) + (static_cast<Real>(2.8333333333333335) * tb88)) + (static_cast<Real>(-0.08333333333333333) * tb100))));
                                const auto tb102 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb8) + (static_cast<Real>(-0.14634146341463414) * tb56)) + (static_cast<Real>(-0.014634146341463415) * tb67)) + (static_cast<Real>(-0.07317073170731707) * tb78)) + (static_cast<Real>(0.07317073170731707) * tb89)) + (static_cast<Real>(0.14634146341463414) * tb101))));
                                const auto tb103 = (-(tb82 * tb84));
                                const auto tb104 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb19) + (static_cast<Real>(0.21296296296296297) * tb47)) + (static_cast<Real>(-7.229629629629629) * tb58)) + (static_cast<Real>(5.7592592592592595) * tb69)) + (static_cast<Real>(-0.31666666666666665) * tb80)) + (static_cast<Real>(2.8333333333333335) * tb91)) + (static_cast<Real>(-0.08333333333333333) * tb103))));
                                const auto tb105 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb10) + (static_cast<Real>(-0.14634146341463414) * tb59)) + (static_cast<Real>(-0.014634146341463415) * tb70)) + (static_cast<Real>(-0.07317073170731707) * tb81)) + (static_cast<Real>(0.07317073170731707) * tb92)) + (static_cast<Real>(0.14634146341463414) * tb104))));
                                const auto tb106 = (((tb99 * tb99) + (tb102 * tb102)) + (tb105 * tb105));
                                const auto tb107 = (static_cast<Real>(1.0) / (tb106 * hk::math::sqrt(tb106)));
                                const auto tb108 = (-(tb99 * tb107));
                                const auto tb109 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb6) + (static_cast<Real>(-2.0792682926829267) * tb24)) + (static_cast<Real>(4.3863414634146345) * tb41)) + (static_cast<Real>(-3.524390243902439) * tb52)) + (static_cast<Real>(0.5348780487804878) * tb63)) + (static_cast<Real>(0.6219512195121951) * tb74)) + (static_cast<Real>(0.20121951219512196) * tb85)) + (static_cast<Real>(0.2926829268292683) * tb96)) + (static_cast<Real>(1.0) * tb108))));
                                const auto tb110 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb53) + (static_cast<Real>(0.2571428571428571) * tb64)) + (static_cast<Real>(0.2571428571428571) * tb75)) + (static_cast<Real>(0.03214285714285714) * tb86)) + (static_cast<Real>(0.03214285714285714) * tb98)) + (static_cast<Real>(0.04880952380952381) * tb97)) + (static_cast<Real>(0.04880952380952381) * tb109))));
                                const auto tb111 = (-(tb90 * tb95));
                                const auto tb112 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb16) + (static_cast<Real>(-0.14634146341463414) * tb66)) + (static_cast<Real>(-0.014634146341463415) * tb77)) + (static_cast<Real>(-0.07317073170731707) * tb88)) + (static_cast<Real>(0.07317073170731707) * tb100)) + (static_cast<Real>(0.14634146341463414) * tb111))));
                                const auto tb113 = (-(tb102 * tb107));
                                const auto tb114 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb16) + (static_cast<Real>(-2.0792682926829267) * tb44)) + (static_cast<Real>(4.3863414634146345) * tb55)) + (static_cast<Real>(-3.524390243902439) * tb66)) + (static_cast<Real>(0.5348780487804878) * tb77)) + (static_cast<Real>(0.6219512195121951) * tb88)) + (static_cast<Real>(0.20121951219512196) * tb100)) + (static_cast<Real>(0.2926829268292683) * tb111)) + (static_cast<Real>(1.0) * tb113))));
                                const auto tb115 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb56) + (static_cast<Real>(0.2571428571428571) * tb67)) + (static_cast<Real>(0.2571428571428571) * tb78)) + (static_cast<Real>(0.03214285714285714) * tb89)) + (static_cast<Real>(0.03214285714285714) * tb101)) + (static_cast<Real>(0.04880952380952381) * tb112)) + (static_cast<Real>(0.04880952380952381) * tb114))));
                                const auto tb116 = (-(tb93 * tb95));
                                const auto tb117 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb19) + (static_cast<Real>(-0.14634146341463414) * tb69)) + (static_cast<Real>(-0.014634146341463415) * tb80)) + (static_cast<Real>(-0.07317073170731707) * tb91)) + (static_cast<Real>(0.07317073170731707) * tb103)) + (static_cast<Real>(0.14634146341463414) * tb116))));
                                const auto tb118 = (-(tb105 * tb107));
                                const auto tb119 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb19) + (static_cast<Real>(-2.0792682926829267) * tb47)) + (static_cast<Real>(4.3863414634146345) * tb58)) + (static_cast<Real>(-3.524390243902439) * tb69)) + (static_cast<Real>(0.5348780487804878) * tb80)) + (static_cast<Real>(0.6219512195121951) * tb91)) + (static_cast<Real>(0.20121951219512196) * tb103)) + (static_cast<Real>(0.2926829268292683) * tb116)) + (static_cast<Real>(1.0) * tb118))));
                                const auto tb120 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb59) + (static_cast<Real>(0.2571428571428571) * tb70)) + (static_cast<Real>(0.2571428571428571) * tb81)) + (static_cast<Real>(0.03214285714285714) * tb92)) + (static_cast<Real>(0.03214285714285714) * tb104)) + (static_cast<Real>(0.04880952380952381) * tb117)) + (static_cast<Real>(0.04880952380952381) * tb119))));
                                const auto tb121 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb3) + (static_cast<Real>(-2.0792682926829267) * tb31)) + (static_cast<Real>(4.3863414634146345) * tb42)) + (static_cast<Real>(-3.6707317073170733) * tb53)) + (static_cast<Real>(0.5202439024390244) * tb64)) + (static_cast<Real>(0.5487804878048781) * tb75)) + (static_cast<Real>(0.27439024390243905) * tb86)) + (static_cast<Real>(0.43902439024390244) * tb98))));
                                const auto tb122 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb8) + (static_cast<Real>(-2.0792682926829267) * tb34)) + (static_cast<Real>(4.3863414634146345) * tb45)) + (static_cast<Real>(-3.6707317073170733) * tb56)) + (static_cast<Real>(0.5202439024390244) * tb67)) + (static_cast<Real>(0.5487804878048781) * tb78)) + (static_cast<Real>(0.27439024390243905) * tb89)) + (static_cast<Real>(0.43902439024390244) * tb101))));
                                const auto tb123 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb10) + (static_cast<Real>(-2.0792682926829267) * tb37)) + (static_cast<Real>(4.3863414634146345) * tb48)) + (static_cast<Real>(-3.6707317073170733) * tb59)) + (static_cast<Real>(0.5202439024390244) * tb70)) + (static_cast<Real>(0.5487804878048781) * tb81)) + (static_cast<Real>(0.27439024390243905) * tb92)) + (static_cast<Real>(0.43902439024390244) * tb104))));
                                const auto tb124 = (((tb121 * tb121) + (tb122 * tb122)) + (tb123 * tb123));
                                const auto tb125 = (static_cast<Real>(1.0) / (tb124 * hk::math::sqrt(tb124)));
                                const auto tb126 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb3) + (static_cast<Real>(-2.0792682926829267) * tb31)) + (static_cast<Real>(4.3863414634146345) * tb42)) + (static_cast<Real>(-3.524390243902439) * tb53)) + (static_cast<Real>(0.5348780487804878) * tb64)) + (static_cast<Real>(0.6219512195121951) * tb75)) + (static_cast<Real>(0.20121951219512196) * tb86)) + (static_cast<Real>(0.2926829268292683) * tb98)) + (static_cast<Real>(1.0) * tb97))));
                                const auto tb127 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb8) + (static_cast<Real>(-2.0792682926829267) * tb34)) + (static_cast<Real>(4.3863414634146345) * tb45)) + (static_cast<Real>(-3.524390243902439) * tb56)) + (static_cast<Real>(0.5348780487804878) * tb67)) + (static_cast<Real>(0.6219512195121951) * tb78)) + (static_cast<Real>(0.20121951219512196) * tb89)) + (static_cast<Real>(0.2926829268292683) * tb101)) + (static_cast<Real>(1.0) * tb112))));
                                const auto tb128 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb10) + (static_cast<Real>(-2.0792682926829267) * tb37)) + (static_cast<Real>(4.3863414634146345) * tb48)) + (static_cast<Real>(-3.524390243902439) * tb59)) + (static_cast<Real>(0.5348780487804878) * tb70)) + (static_cast<Real>(0.6219512195121951) * tb81)) + (static_cast<Real>(0.20121951219512196) * tb92)) + (static_cast<Real>(0.2926829268292683) * tb104)) + (static_cast<Real>(1.0) * tb117))));
                                const auto tb129 = (((tb126 * tb126) + (tb127 * tb127)) + (tb128 * tb128));
                                const auto tb130 = (static_cast<Real>(1.0) / (tb129 * hk::math::sqrt(tb129)));
                                const auto tb131 = (-(tb126 * tb130));
                                const auto tb132 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb52) + (static_cast<Real>(0.2571428571428571) * tb63)) + (static_cast<Real>(0.2571428571428571) * tb74)) + (static_cast<Real>(0.03214285714285714) * tb85)) + (static_cast<Real>(0.03214285714285714) * tb96)) + (static_cast<Real>(0.04880952380952381) * tb108)) + (static_cast<Real>(0.04880952380952381) * tb131))));
                                const auto tb133 = (-(tb127 * tb130));
                                const auto tb134 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb66) + (static_cast<Real>(0.2571428571428571) * tb77)) + (static_cast<Real>(0.2571428571428571) * tb88)) + (static_cast<Real>(0.03214285714285714) * tb100)) + (static_cast<Real>(0.03214285714285714) * tb111)) + (static_cast<Real>(0.04880952380952381) * tb113)) + (static_cast<Real>(0.04880952380952381) * tb133))));
                                const auto tb135 = (-(tb128 * tb130));
                                const auto tb136 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb69) + (static_cast<Real>(0.2571428571428571) * tb80)) + (static_cast<Real>(0.2571428571428571) * tb91)) + (static_cast<Real>(0.03214285714285714) * tb103)) + (static_cast<Real>(0.03214285714285714) * tb116)) + (static_cast<Real>(0.04880952380952381) * tb118)) + (static_cast<Real>(0.04880952380952381) * tb135))));
                                const auto tb137 = hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax((hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb3) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb6) + (static_cast<Real>(-2.0792682926829267) * tb24)) + (static_cast<Real>(4.3863414634146345) * tb41)) + (static_cast<Real>(-3.6707317073170733) * tb52)) + (static_cast<Real>(0.5202439024390244) * tb63)) + (static_cast<Real>(0.5487804878048781) * tb74)) + (static_cast<Real>(0.27439024390243905) * tb85)) + (static_cast<Real>(0.43902439024390244) * tb96)))))) + (static_cast<Real>(-1.0) * tb97)) + (static_cast<Real>(-1.0) * tb109)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb110), hk::math::abs(hawk_v73_0_s.eval<0>(i)))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb8) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb16) + (static_cast<Real>(-2.0792682926829267) * tb44)) + (static_cast<Real>(4.3863414634146345) * tb55)) + (static_cast<Real>(-3.6707317073170733) * tb66)) + (static_cast<Real>(0.5202439024390244) * tb77)) + (static_cast<Real>(0.5487804878048781) * tb88)) + (static_cast<Real>(0.27439024390243905) * tb100)) + (static_cast<Real>(0.43902439024390244) * tb111)))))) + (static_cast<Real>(-1.0) * tb112)) + (static_cast<Real>(-1.0) * tb114)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb115), hk::math::abs(hawk_v73_0_s.eval<1>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb10) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb19) + (static_cast<Real>(-2.0792682926829267) * tb47)) + (static_cast<Real>(4.3863414634146345) * tb58)) + (static_cast<Real>(-3.6707317073170733) * tb69)) + (static_cast<Real>(0.5202439024390244) * tb80)) + (static_cast<Real>(0.5487804878048781) * tb91)) + (static_cast<Real>(0.27439024390243905) * tb103)) + (static_cast<Real>(0.43902439024390244) * tb116)))))) + (static_cast<Real>(-1.0) * tb117)) + (static_cast<Real>(-1.0) * tb119)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb120), hk::math::abs(hawk_v73_0_s.eval<2>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb6) + (static_cast<Real>(1.0) * (-(tb121 * tb125)))) + (static_cast<Real>(-1.0) * tb108)) + (static_cast<Real>(-1.0) * tb131)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb132), hk::math::abs(hawk_v73_0_s.eval<3>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb16) + (static_cast<Real>(1.0) * (-(tb122 * tb125)))) + (static_cast<Real>(-1.0) * tb113)) + (static_cast<Real>(-1.0) * tb133)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb134), hk::math::abs(hawk_v73_0_s.eval<4>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb19) + (static_cast<Real>(1.0) * (-(tb123 * tb125)))) + (static_cast<Real>(-1.0) * tb118)) + (static_cast<Real>(-1.0) * tb135)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb136), hk::math::abs(hawk_v73_0_s.eval<5>(i)))))));
                                const auto tb138 = (tb137 < static_cast<Real>(1.0));
                                const auto tb139 = hk::Item<Real, 6>{tb110, tb115, tb120, tb132, tb134, tb136};
                                const auto hz0 = hk::constant<hk::extents<>>(tb138);
                                const auto tb140 = (tb1 ? psc_t_end_i : (hawk_v73_1_t + tb2));
                                const auto tb141 = (tb138 ? tb140 : hawk_v73_1_t);
                                const auto tb142 = hk::math::fmin(static_cast<Real>(5.0), hk::math::fmax(static_cast<Real>(0.2), (static_cast<Real>(0.9) * (static_cast<Real>(1.0) / hk::math::sqrt(hk::math::sqrt(hk::math::sqrt(tb137)))))));
                                const auto tb143 = (tb138 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                                const auto tb144 = (tb138 ? static_cast<Real>(0.0) : static_cast<Real>(1.0));
                                const auto tb145 = (tb141 >= psc_t_end_i);
                                const hk::Item<Real, 6> hawk_n73_0 = hk::select(hz0, tb139, hawk_v73_0_s);
                                const Real hawk_n73_1 = tb141;
                                const Real hawk_n73_2 = (tb2 * tb142);
                                const Real hawk_n73_3 = (hawk_v73_3_n_acc + tb143);
                                const Real hawk_n73_4 = (hawk_v73_4_n_rej + tb144);
                                const Real hawk_n73_5 = (tb145 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                                const bool hawk_x73 = tb145;
                hk_c0 = hawk_n73_0;
                hk_c1 = hawk_n73_1;
                hk_c2 = hawk_n73_2;
                hk_c3 = hawk_n73_3;
                hk_c4 = hawk_n73_4;
                hk_c5 = hawk_n73_5;
                ++hk_trip;
                if (hawk_x73 || hk_trip >= hk_budget) {
                    const hk::Item<Real, 6> hawk_v73_0_s = hk_c0;
                    const Real hawk_v73_1_t = hk_c1;
                    const Real hawk_v73_2_h = hk_c2;
                    const Real hawk_v73_3_n_acc = hk_c3;
                    const Real hawk_v73_4_n_rej = hk_c4;
                    const Real hawk_v73_5_finished = hk_c5;
                    (void)hawk_v73_0_s;
                    (void)hawk_v73_1_t;
                    (void)hawk_v73_2_h;
                    (void)hawk_v73_3_n_acc;
                    (void)hawk_v73_4_n_rej;
                    (void)hawk_v73_5_finished;
                        mut_s[i] = hawk_v73_0_s;
                            mut_t[i] = hawk_v73_1_t;
                            mut_h[i] = hawk_v73_2_h;
                            mut_n_acc[i] = hawk_v73_3_n_acc;
                            mut_n_rej[i] = hawk_v73_4_n_rej;
                            if (!trm_terminated[i].eval() && (hawk_v73_5_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; ++hk_fin; }
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

extern "C" __global__ void __launch_bounds__(256) orbit_range(
    hk::abi::ScalarHandle p_mut_h,
    hk::abi::ScalarHandle p_mut_n_acc,
    hk::abi::ScalarHandle p_mut_n_rej,
    hk::abi::GRefMirror p_mut_s,
    hk::abi::ScalarHandle p_mut_t,
    hk::abi::ScalarHandle p_psc_t_end,
    hk::abi::ScalarHandle p_lut_finished_count,
    hk::abi::ScalarHandle p_lut_fused_steps,
    hk::abi::ScalarHandle p_trm_terminated,
    long long base,
    long long count,
    long long nSamples,
    unsigned int* hawk_steps,
    unsigned long long* hawk_stepsum)
{
    const hk::ScalarOut<Real> mut_h(p_mut_h);
    (void)mut_h;
    const hk::ScalarOut<Real> mut_n_acc(p_mut_n_acc);
    (void)mut_n_acc;
    const hk::ScalarOut<Real> mut_n_rej(p_mut_n_rej);
    (void)mut_n_rej;
    const hk::VecOut<Real, 6> mut_s(p_mut_s);
    (void)mut_s;
    const hk::ScalarOut<Real> mut_t(p_mut_t);
    (void)mut_t;
    const hk::ScalarIn<Real> psc_t_end(p_psc_t_end);
    (void)psc_t_end;
    const hk::ScalarIn<std::uint32_t> lut_finished_count(p_lut_finished_count);
    (void)lut_finished_count;
    const hk::ScalarIn<Int> lut_fused_steps(p_lut_fused_steps);
    (void)lut_fused_steps;
    const hk::MaskView trm_terminated(p_trm_terminated);
    (void)trm_terminated;
    const hk::MaskView trm_terminated_w(p_trm_terminated);
    (void)trm_terminated_w;
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
            const auto mut_h_i = mut_h[i].get()();
            const auto psc_t_end_i = psc_t_end[i].eval();
            const auto mut_t_i = mut_t[i].get()();
            const auto t3 = (psc_t_end_i - mut_t_i);
            const auto t4 = (mut_h_i >= t3);
            const auto t5 = (t4 ? t3 : mut_h_i);
            const auto t7 = (t5 * static_cast<Real>(0.04880952380952381));
            const auto mut_s_i = mut_s[i].get();
            const auto t10 = mut_s_i.eval<3>(i);
            const auto t13 = mut_s_i.eval<0>(i);
            const auto t15 = mut_s_i.eval<1>(i);
            const auto t18 = mut_s_i.eval<2>(i);
            const auto t20 = (((t13 * t13) + (t15 * t15)) + (t18 * t18));
            const auto t23 = (static_cast<Real>(1.0) / (t20 * hk::math::sqrt(t20)));
            const auto t25 = (-(t13 * t23));
            const auto t37 = (t13 + (t5 * (static_cast<Real>(0.07407407407407407) * t10)));
            const auto t39 = mut_s_i.eval<4>(i);
            const auto t42 = (t15 + (t5 * (static_cast<Real>(0.07407407407407407) * t39)));
            const auto t45 = mut_s_i.eval<5>(i);
            const auto t48 = (t18 + (t5 * (static_cast<Real>(0.07407407407407407) * t45)));
            const auto t50 = (((t37 * t37) + (t42 * t42)) + (t48 * t48));
            const auto t53 = (static_cast<Real>(1.0) / (t50 * hk::math::sqrt(t50)));
            const auto t59 = (t10 + (t5 * ((static_cast<Real>(0.027777777777777776) * t25) + (static_cast<Real>(0.08333333333333333) * (-(t37 * t53))))));
            const auto t63 = (t13 + (t5 * ((static_cast<Real>(0.041666666666666664) * t10) + (static_cast<Real>(0.125) * t59))));
            const auto t67 = (-(t15 * t23));
            const auto t74 = (t39 + (t5 * ((static_cast<Real>(0.027777777777777776) * t67) + (static_cast<Real>(0.08333333333333333) * (-(t42 * t53))))));
            const auto t78 = (t15 + (t5 * ((static_cast<Real>(0.041666666666666664) * t39) + (static_cast<Real>(0.125) * t74))));
            const auto t83 = (-(t18 * t23));
            const auto t90 = (t45 + (t5 * ((static_cast<Real>(0.027777777777777776) * t83) + (static_cast<Real>(0.08333333333333333) * (-(t48 * t53))))));
            const auto t94 = (t18 + (t5 * ((static_cast<Real>(0.041666666666666664) * t45) + (static_cast<Real>(0.125) * t90))));
            const auto t96 = (((t63 * t63) + (t78 * t78)) + (t94 * t94));
            const auto t99 = (static_cast<Real>(1.0) / (t96 * hk::math::sqrt(t96)));
            const auto t101 = (-(t63 * t99));
            const auto t102 = (static_cast<Real>(-2.0792682926829267) * t101);
            const auto t119 = (t13 + (t5 * ((static_cast<Real>(0.027777777777777776) * t10) + (static_cast<Real>(0.08333333333333333) * (t10 + (t5 * (static_cast<Real>(0.07407407407407407) * t25)))))));
            const auto t128 = (t15 + (t5 * ((static_cast<Real>(0.027777777777777776) * t39) + (static_cast<Real>(0.08333333333333333) * (t39 + (t5 * (static_cast<Real>(0.07407407407407407) * t67)))))));
            const auto t138 = (t18 + (t5 * ((static_cast<Real>(0.027777777777777776) * t45) + (static_cast<Real>(0.08333333333333333) * (t45 + (t5 * (static_cast<Real>(0.07407407407407407) * t83)))))));
            const auto t140 = (((t119 * t119) + (t128 * t128)) + (t138 * t138));
            const auto t143 = (static_cast<Real>(1.0) / (t140 * hk::math::sqrt(t140)));
            const auto t145 = (-(t119 * t143));
            const auto t149 = (t10 + (t5 * ((static_cast<Real>(0.041666666666666664) * t25) + (static_cast<Real>(0.125) * t145))));
            const auto t153 = (t13 + (t5 * (((static_cast<Real>(0.4166666666666667) * t10) + (static_cast<Real>(-1.5625) * t59)) + (static_cast<Real>(1.5625) * t149))));
            const auto t160 = (-(t128 * t143));
            const auto t164 = (t39 + (t5 * ((static_cast<Real>(0.041666666666666664) * t67) + (static_cast<Real>(0.125) * t160))));
            const auto t168 = (t15 + (t5 * (((static_cast<Real>(0.4166666666666667) * t39) + (static_cast<Real>(-1.5625) * t74)) + (static_cast<Real>(1.5625) * t164))));
            const auto t176 = (-(t138 * t143));
            const auto t180 = (t45 + (t5 * ((static_cast<Real>(0.041666666666666664) * t83) + (static_cast<Real>(0.125) * t176))));
            const auto t184 = (t18 + (t5 * (((static_cast<Real>(0.4166666666666667) * t45) + (static_cast<Real>(-1.5625) * t90)) + (static_cast<Real>(1.5625) * t180))));
            const auto t186 = (((t153 * t153) + (t168 * t168)) + (t184 * t184));
            const auto t189 = (static_cast<Real>(1.0) / (t186 * hk::math::sqrt(t186)));
            const auto t191 = (-(t153 * t189));
            const auto t192 = (static_cast<Real>(4.3863414634146345) * t191);
            const auto t207 = (t10 + (t5 * (((static_cast<Real>(0.4166666666666667) * t25) + (static_cast<Real>(-1.5625) * t145)) + (static_cast<Real>(1.5625) * t101))));
            const auto t211 = (t13 + (t5 * (((static_cast<Real>(0.05) * t10) + (static_cast<Real>(0.25) * t149)) + (static_cast<Real>(0.2) * t207))));
            const auto t220 = (-(t78 * t99));
            const auto t224 = (t39 + (t5 * (((static_cast<Real>(0.4166666666666667) * t67) + (static_cast<Real>(-1.5625) * t160)) + (static_cast<Real>(1.5625) * t220))));
            const auto t228 = (t15 + (t5 * (((static_cast<Real>(0.05) * t39) + (static_cast<Real>(0.25) * t164)) + (static_cast<Real>(0.2) * t224))));
            const auto t238 = (-(t94 * t99));
            const auto t242 = (t45 + (t5 * (((static_cast<Real>(0.4166666666666667) * t83) + (static_cast<Real>(-1.5625) * t176)) + (static_cast<Real>(1.5625) * t238))));
            const auto t246 = (t18 + (t5 * (((static_cast<Real>(0.05) * t45) + (static_cast<Real>(0.25) * t180)) + (static_cast<Real>(0.2) * t242))));
            const auto t248 = (((t211 * t211) + (t228 * t228)) + (t246 * t246));
            const auto t251 = (static_cast<Real>(1.0) / (t248 * hk::math::sqrt(t248)));
            const auto t253 = (-(t211 * t251));
            const auto t272 = (t10 + (t5 * (((static_cast<Real>(0.05) * t25) + (static_cast<Real>(0.25) * t101)) + (static_cast<Real>(0.2) * t191))));
            const auto t276 = (t13 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t10) + (static_cast<Real>(1.1574074074074074) * t149)) + (static_cast<Real>(-2.4074074074074074) * t207)) + (static_cast<Real>(2.314814814814815) * t272))));
            const auto t287 = (-(t168 * t189));
            const auto t291 = (t39 + (t5 * (((static_cast<Real>(0.05) * t67) + (static_cast<Real>(0.25) * t220)) + (static_cast<Real>(0.2) * t287))));
            const auto t295 = (t15 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t39) + (static_cast<Real>(1.1574074074074074) * t164)) + (static_cast<Real>(-2.4074074074074074) * t224)) + (static_cast<Real>(2.314814814814815) * t291))));
            const auto t307 = (-(t184 * t189));
            const auto t311 = (t45 + (t5 * (((static_cast<Real>(0.05) * t83) + (static_cast<Real>(0.25) * t238)) + (static_cast<Real>(0.2) * t307))));
            const auto t315 = (t18 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t45) + (static_cast<Real>(1.1574074074074074) * t180)) + (static_cast<Real>(-2.4074074074074074) * t242)) + (static_cast<Real>(2.314814814814815) * t311))));
            const auto t317 = (((t276 * t276) + (t295 * t295)) + (t315 * t315));
            const auto t320 = (static_cast<Real>(1.0) / (t317 * hk::math::sqrt(t317)));
            const auto t322 = (-(t276 * t320));
            const auto t343 = (t10 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t25) + (static_cast<Real>(1.1574074074074074) * t101)) + (static_cast<Real>(-2.4074074074074074) * t191)) + (static_cast<Real>(2.314814814814815) * t253))));
            const auto t347 = (t13 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t10) + (static_cast<Real>(0.27111111111111114) * t207)) + (static_cast<Real>(-0.2222222222222222) * t272)) + (static_cast<Real>(0.014444444444444444) * t343))));
            const auto t360 = (-(t228 * t251));
            const auto t364 = (t39 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t67) + (static_cast<Real>(1.1574074074074074) * t220)) + (static_cast<Real>(-2.4074074074074074) * t287)) + (static_cast<Real>(2.314814814814815) * t360))));
            const auto t368 = (t15 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t39) + (static_cast<Real>(0.27111111111111114) * t224)) + (static_cast<Real>(-0.2222222222222222) * t291)) + (static_cast<Real>(0.014444444444444444) * t364))));
            const auto t382 = (-(t246 * t251));
            const auto t386 = (t45 + (t5 * ((((static_cast<Real>(-0.23148148148148148) * t83) + (static_cast<Real>(1.1574074074074074) * t238)) + (static_cast<Real>(-2.4074074074074074) * t307)) + (static_cast<Real>(2.314814814814815) * t382))));
            const auto t390 = (t18 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t45) + (static_cast<Real>(0.27111111111111114) * t242)) + (static_cast<Real>(-0.2222222222222222) * t311)) + (static_cast<Real>(0.014444444444444444) * t386))));
            const auto t392 = (((t347 * t347) + (t368 * t368)) + (t390 * t390));
            const auto t395 = (static_cast<Real>(1.0) / (t392 * hk::math::sqrt(t392)));
            const auto t397 = (-(t347 * t395));
            const auto t424 = (t10 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t25) + (static_cast<Real>(0.27111111111111114) * t191)) + (static_cast<Real>(-0.2222222222222222) * t253)) + (static_cast<Real>(0.014444444444444444) * t322))));
            const auto t428 = (t13 + (t5 * ((((((static_cast<Real>(2.0) * t10) + (static_cast<Real>(-8.833333333333334) * t149)) + (static_cast<Real>(15.644444444444444) * t207)) + (static_cast<Real>(-11.88888888888889) * t272)) + (static_cast<Real>(0.7444444444444445) * t343)) + (static_cast<Real>(3.0) * t424))));
            const auto t445 = (-(t295 * t320));
            const auto t449 = (t39 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t67) + (static_cast<Real>(0.27111111111111114) * t287)) + (static_cast<Real>(-0.2222222222222222) * t360)) + (static_cast<Real>(0.014444444444444444) * t445))));
            const auto t453 = (t15 + (t5 * ((((((static_cast<Real>(2.0) * t39) + (static_cast<Real>(-8.833333333333334) * t164)) + (static_cast<Real>(15.644444444444444) * t224)) + (static_cast<Real>(-11.88888888888889) * t291)) + (static_cast<Real>(0.7444444444444445) * t364)) + (static_cast<Real>(3.0) * t449))));
            const auto t471 = (-(t315 * t320));
            const auto t475 = (t45 + (t5 * ((((static_cast<Real>(0.10333333333333333) * t83) + (static_cast<Real>(0.27111111111111114) * t307)) + (static_cast<Real>(-0.2222222222222222) * t382)) + (static_cast<Real>(0.014444444444444444) * t471))));
            const auto t479 = (t18 + (t5 * ((((((static_cast<Real>(2.0) * t45) + (static_cast<Real>(-8.833333333333334) * t180)) + (static_cast<Real>(15.644444444444444) * t242)) + (static_cast<Real>(-11.88888888888889) * t311)) + (static_cast<Real>(0.7444444444444445) * t386)) + (static_cast<Real>(3.0) * t475))));
            const auto t481 = (((t428 * t428) + (t453 * t453)) + (t479 * t479));
            const auto t484 = (static_cast<Real>(1.0) / (t481 * hk::math::sqrt(t481)));
            const auto t486 = (-(t428 * t484));
            const auto t520 = (t10 + (t5 * ((((((static_cast<Real>(2.0) * t25) + (static_cast<Real>(-8.833333333333334) * t101)) + (static_cast<Real>(15.644444444444444) * t191)) + (static_cast<Real>(-11.88888888888889) * t253)) + (static_cast<Real>(0.7444444444444445) * t322)) + (static_cast<Real>(3.0) * t397))));
            const auto t524 = (t13 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t10) + (static_cast<Real>(0.21296296296296297) * t149)) + (static_cast<Real>(-7.229629629629629) * t207)) + (static_cast<Real>(5.7592592592592595) * t272)) + (static_cast<Real>(-0.31666666666666665) * t343)) + (static_cast<Real>(2.8333333333333335) * t424)) + (static_cast<Real>(-0.08333333333333333) * t520))));
            const auto t547 = (-(t368 * t395));
            const auto t551 = (t39 + (t5 * ((((((static_cast<Real>(2.0) * t67) + (static_cast<Real>(-8.833333333333334) * t220)) + (static_cast<Real>(15.644444444444444) * t287)) + (static_cast<Real>(-11.88888888888889) * t360)) + (static_cast<Real>(0.7444444444444445) * t445)) + (static_cast<Real>(3.0) * t547))));
            const auto t555 = (t15 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t39) + (static_cast<Real>(0.21296296296296297) * t164)) + (static_cast<Real>(-7.229629629629629) * t224)) + (static_cast<Real>(5.7592592592592595) * t291)) + (static_cast<Real>(-0.31666666666666665) * t364)) + (static_cast<Real>(2.8333333333333335) * t449)) + (static_cast<Real>(-0.08333333333333333) * t551))));
            const auto t579 = (-(t390 * t395));
            const auto t583 = (t45 + (t5 * ((((((static_cast<Real>(2.0) * t83) + (static_cast<Real>(-8.833333333333334) * t238)) + (static_cast<Real>(15.644444444444444) * t307)) + (static_cast<Real>(-11.88888888888889) * t382)) + (static_cast<Real>(0.7444444444444445) * t471)) + (static_cast<Real>(3.0) * t579))));
            const auto t587 = (t18 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t45) + (static_cast<Real>(0.21296296296296297) * t180)) + (static_cast<Real>(-7.229629629629629) * t242)) + (static_cast<Real>(5.7592592592592595) * t311)) + (static_cast<Real>(-0.31666666666666665) * t386)) + (static_cast<Real>(2.8333333333333335) * t475)) + (static_cast<Real>(-0.08333333333333333) * t583))));
            const auto t589 = (((t524 * t524) + (t555 * t555)) + (t587 * t587));
            const auto t592 = (static_cast<Real>(1.0) / (t589 * hk::math::sqrt(t589)));
            const auto t594 = (-(t524 * t592));
            const auto t620 = (t10 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t25) + (static_cast<Real>(-0.14634146341463414) * t253)) + (static_cast<Real>(-0.014634146341463415) * t322)) + (static_cast<Real>(-0.07317073170731707) * t397)) + (static_cast<Real>(0.07317073170731707) * t486)) + (static_cast<Real>(0.14634146341463414) * t594))));
            const auto t665 = (t10 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t25) + (static_cast<Real>(0.21296296296296297) * t101)) + (static_cast<Real>(-7.229629629629629) * t191)) + (static_cast<Real>(5.7592592592592595) * t253)) + (static_cast<Real>(-0.31666666666666665) * t322)) + (static_cast<Real>(2.8333333333333335) * t397)) + (static_cast<Real>(-0.08333333333333333) * t486))));
            const auto t669 = (t13 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t10) + (static_cast<Real>(-0.14634146341463414) * t272)) + (static_cast<Real>(-0.014634146341463415) * t343)) + (static_cast<Real>(-0.07317073170731707) * t424)) + (static_cast<Real>(0.07317073170731707) * t520)) + (static_cast<Real>(0.14634146341463414) * t665))));
            const auto t692 = (-(t453 * t484));
            const auto t696 = (t39 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t67) + (static_cast<Real>(0.21296296296296297) * t220)) + (static_cast<Real>(-7.229629629629629) * t287)) + (static_cast<Real>(5.7592592592592595) * t360)) + (static_cast<Real>(-0.31666666666666665) * t445)) + (static_cast<Real>(2.8333333333333335) * t547)) + (static_cast<Real>(-0.08333333333333333) * t692))));
            const auto t700 = (t15 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t39) + (static_cast<Real>(-0.14634146341463414) * t291)) + (static_cast<Real>(-0.014634146341463415) * t364)) + (static_cast<Real>(-0.07317073170731707) * t449)) + (static_cast<Real>(0.07317073170731707) * t551)) + (static_cast<Real>(0.14634146341463414) * t696))));
            const auto t724 = (-(t479 * t484));
            const auto t728 = (t45 + (t5 * (((((((static_cast<Real>(-0.8425925925925926) * t83) + (static_cast<Real>(0.21296296296296297) * t238)) + (static_cast<Real>(-7.229629629629629) * t307)) + (static_cast<Real>(5.7592592592592595) * t382)) + (static_cast<Real>(-0.31666666666666665) * t471)) + (static_cast<Real>(2.8333333333333335) * t579)) + (static_cast<Real>(-0.08333333333333333) * t724))));
            const auto t732 = (t18 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t45) + (static_cast<Real>(-0.14634146341463414) * t311)) + (static_cast<Real>(-0.014634146341463415) * t386)) + (static_cast<Real>(-0.07317073170731707) * t475)) + (static_cast<Real>(0.07317073170731707) * t583)) + (static_cast<Real>(0.14634146341463414) * t728))));
            const auto t734 = (((t669 * t669) + (t700 * t700)) + (t732 * t732));
            const auto t737 = (static_cast<Real>(1.0) / (t734 * hk::math::sqrt(t734)));
            const auto t739 = (-(t669 * t737));
            const auto t743 = (t10 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t25) + t102) + t192) + (static_cast<Real>(-3.524390243902439) * t253)) + (static_cast<Real>(0.5348780487804878) * t322)) + (static_cast<Real>(0.6219512195121951) * t397)) + (static_cast<Real>(0.20121951219512196) * t486)) + (static_cast<Real>(0.2926829268292683) * t594)) + (static_cast<Real>(1.0) * t739))));
            const auto t766 = (t13 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t272) + (static_cast<Real>(0.2571428571428571) * t343)) + (static_cast<Real>(0.2571428571428571) * t424)) + (static_cast<Real>(0.03214285714285714) * t520)) + (static_cast<Real>(0.03214285714285714) * t665)) + (static_cast<Real>(0.04880952380952381) * t620)) + (static_cast<Real>(0.04880952380952381) * t743))));
            const auto t775 = (static_cast<Real>(-2.0792682926829267) * t220);
            const auto t777 = (static_cast<Real>(4.3863414634146345) * t287);
            const auto t788 = (-(t555 * t592));
            const auto t807 = (t39 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t67) + (static_cast<Real>(-0.14634146341463414) * t360)) + (static_cast<Real>(-0.014634146341463415) * t445)) + (static_cast<Real>(-0.07317073170731707) * t547)) + (static_cast<Real>(0.07317073170731707) * t692)) + (static_cast<Real>(0.14634146341463414) * t788))));
            const auto t824 = (-(t700 * t737));
            const auto t828 = (t39 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t67) + t775) + t777) + (static_cast<Real>(-3.524390243902439) * t360)) + (static_cast<Real>(0.5348780487804878) * t445)) + (static_cast<Real>(0.6219512195121951) * t547)) + (static_cast<Real>(0.20121951219512196) * t692)) + (static_cast<Real>(0.2926829268292683) * t788)) + (static_cast<Real>(1.0) * t824))));
            const auto t847 = (t15 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t291) + (static_cast<Real>(0.2571428571428571) * t364)) + (static_cast<Real>(0.2571428571428571) * t449)) + (static_cast<Real>(0.03214285714285714) * t551)) + (static_cast<Real>(0.03214285714285714) * t696)) + (static_cast<Real>(0.04880952380952381) * t807)) + (static_cast<Real>(0.04880952380952381) * t828))));
            const auto t857 = (static_cast<Real>(-2.0792682926829267) * t238);
            const auto t859 = (static_cast<Real>(4.3863414634146345) * t307);
            const auto t870 = (-(t587 * t592));
            const auto t889 = (t45 + (t5 * ((((((static_cast<Real>(0.014634146341463415) * t83) + (static_cast<Real>(-0.14634146341463414) * t382)) + (static_cast<Real>(-0.014634146341463415) * t471)) + (static_cast<Real>(-0.07317073170731707) * t579)) + (static_cast<Real>(0.07317073170731707) * t724)) + (static_cast<Real>(0.14634146341463414) * t870))));
            const auto t906 = (-(t732 * t737));
            const auto t910 = (t45 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t83) + t857) + t859) + (static_cast<Real>(-3.524390243902439) * t382)) + (static_cast<Real>(0.5348780487804878) * t471)) + (static_cast<Real>(0.6219512195121951) * t579)) + (static_cast<Real>(0.20121951219512196) * t724)) + (static_cast<Real>(0.2926829268292683) * t870)) + (static_cast<Real>(1.0) * t906))));
            const auto t929 = (t18 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t311) + (static_cast<Real>(0.2571428571428571) * t386)) + (static_cast<Real>(0.2571428571428571) * t475)) + (static_cast<Real>(0.03214285714285714) * t583)) + (static_cast<Real>(0.03214285714285714) * t728)) + (static_cast<Real>(0.04880952380952381) * t889)) + (static_cast<Real>(0.04880952380952381) * t910))));
            const auto t939 = (static_cast<Real>(-2.0792682926829267) * t149);
            const auto t941 = (static_cast<Real>(4.3863414634146345) * t207);
            const auto t954 = (t13 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t10) + t939) + t941) + (static_cast<Real>(-3.6707317073170733) * t272)) + (static_cast<Real>(0.5202439024390244) * t343)) + (static_cast<Real>(0.5487804878048781) * t424)) + (static_cast<Real>(0.27439024390243905) * t520)) + (static_cast<Real>(0.43902439024390244) * t665))));
            const auto t957 = (static_cast<Real>(-2.0792682926829267) * t164);
            const auto t959 = (static_cast<Real>(4.3863414634146345) * t224);
            const auto t972 = (t15 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t39) + t957) + t959) + (static_cast<Real>(-3.6707317073170733) * t291)) + (static_cast<Real>(0.5202439024390244) * t364)) + (static_cast<Real>(0.5487804878048781) * t449)) + (static_cast<Real>(0.27439024390243905) * t551)) + (static_cast<Real>(0.43902439024390244) * t696))));
            const auto t976 = (static_cast<Real>(-2.0792682926829267) * t180);
            const auto t978 = (static_cast<Real>(4.3863414634146345) * t242);
            const auto t991 = (t18 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t45) + t976) + t978) + (static_cast<Real>(-3.6707317073170733) * t311)) + (static_cast<Real>(0.5202439024390244) * t386)) + (static_cast<Real>(0.5487804878048781) * t475)) + (static_cast<Real>(0.27439024390243905) * t583)) + (static_cast<Real>(0.43902439024390244) * t728))));
            const auto t993 = (((t954 * t954) + (t972 * t972)) + (t991 * t991));
            const auto t996 = (static_cast<Real>(1.0) / (t993 * hk::math::sqrt(t993)));
            const auto t1019 = (t13 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t10) + t939) + t941) + (static_cast<Real>(-3.524390243902439) * t272)) + (static_cast<Real>(0.5348780487804878) * t343)) + (static_cast<Real>(0.6219512195121951) * t424)) + (static_cast<Real>(0.20121951219512196) * t520)) + (static_cast<Real>(0.2926829268292683) * t665)) + (static_cast<Real>(1.0) * t620))));
            const auto t1037 = (t15 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t39) + t957) + t959) + (static_cast<Real>(-3.524390243902439) * t291)) + (static_cast<Real>(0.5348780487804878) * t364)) + (static_cast<Real>(0.6219512195121951) * t449)) + (static_cast<Real>(0.20121951219512196) * t551)) + (static_cast<Real>(0.2926829268292683) * t696)) + (static_cast<Real>(1.0) * t807))));
            const auto t1056 = (t18 + (t5 * (((((((((static_cast<Real>(-0.43341463414634146) * t45) + t976) + t978) + (static_cast<Real>(-3.524390243902439) * t311)) + (static_cast<Real>(0.5348780487804878) * t386)) + (static_cast<Real>(0.6219512195121951) * t475)) + (static_cast<Real>(0.20121951219512196) * t583)) + (static_cast<Real>(0.2926829268292683) * t728)) + (static_cast<Real>(1.0) * t889))));
            const auto t1058 = (((t1019 * t1019) + (t1037 * t1037)) + (t1056 * t1056));
            const auto t1061 = (static_cast<Real>(1.0) / (t1058 * hk::math::sqrt(t1058)));
            const auto t1063 = (-(t1019 * t1061));
            const auto t1082 = (t10 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t253) + (static_cast<Real>(0.2571428571428571) * t322)) + (static_cast<Real>(0.2571428571428571) * t397)) + (static_cast<Real>(0.03214285714285714) * t486)) + (static_cast<Real>(0.03214285714285714) * t594)) + (static_cast<Real>(0.04880952380952381) * t739)) + (static_cast<Real>(0.04880952380952381) * t1063))));
            const auto t1098 = (-(t1037 * t1061));
            const auto t1117 = (t39 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t360) + (static_cast<Real>(0.2571428571428571) * t445)) + (static_cast<Real>(0.2571428571428571) * t547)) + (static_cast<Real>(0.03214285714285714) * t692)) + (static_cast<Real>(0.03214285714285714) * t788)) + (static_cast<Real>(0.04880952380952381) * t824)) + (static_cast<Real>(0.04880952380952381) * t1098))));
            const auto t1133 = (-(t1056 * t1061));
            const auto t1152 = (t45 + (t5 * (((((((static_cast<Real>(0.3238095238095238) * t382) + (static_cast<Real>(0.2571428571428571) * t471)) + (static_cast<Real>(0.2571428571428571) * t579)) + (static_cast<Real>(0.03214285714285714) * t724)) + (static_cast<Real>(0.03214285714285714) * t870)) + (static_cast<Real>(0.04880952380952381) * t906)) + (static_cast<Real>(0.04880952380952381) * t1133))));
            const auto t1159 = hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax((hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t10) + (static_cast<Real>(1.0) * (t10 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t25) + t102) + t192) + (static_cast<Real>(-3.6707317073170733) * t253)) + (static_cast<Real>(0.5202439024390244) * t322)) + (static_cast<Real>(0.5487804878048781) * t397)) + (static_cast<Real>(0.27439024390243905) * t486)) + (static_cast<Real>(0.43902439024390244) * t594)))))) + (static_cast<Real>(-1.0) * t620)) + (static_cast<Real>(-1.0) * t743)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t766), hk::math::abs(t13))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t39) + (static_cast<Real>(1.0) * (t39 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t67) + t775) + t777) + (static_cast<Real>(-3.6707317073170733) * t360)) + (static_cast<Real>(0.5202439024390244) * t445)) + (static_cast<Real>(0.5487804878048781) * t547)) + (static_cast<Real>(0.27439024390243905) * t692)) + (static_cast<Real>(0.43902439024390244) * t788)))))) + (static_cast<Real>(-1.0) * t807)) + (static_cast<Real>(-1.0) * t828)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t847), hk::math::abs(t15)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t45) + (static_cast<Real>(1.0) * (t45 + (t5 * ((((((((static_cast<Real>(0.5812195121951219) * t83) + t857) + t859) + (static_cast<Real>(-3.6707317073170733) * t382)) + (static_cast<Real>(0.5202439024390244) * t471)) + (static_cast<Real>(0.5487804878048781) * t579)) + (static_cast<Real>(0.27439024390243905) * t724)) + (static_cast<Real>(0.43902439024390244) * t870)))))) + (static_cast<Real>(-1.0) * t889)) + (static_cast<Real>(-1.0) * t910)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t929), hk::math::abs(t18)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t25) + (static_cast<Real>(1.0) * (-(t954 * t996)))) + (static_cast<Real>(-1.0) * t739)) + (static_cast<Real>(-1.0) * t1063)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t1082), hk::math::abs(t10)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t67) + (static_cast<Real>(1.0) * (-(t972 * t996)))) + (static_cast<Real>(-1.0) * t824)) + (static_cast<Real>(-1.0) * t1098)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t1117), hk::math::abs(t39)))))), (hk::math::abs((t7 * ((((static_cast<Real>(1.0) * t83) + (static_cast<Real>(1.0) * (-(t991 * t996)))) + (static_cast<Real>(-1.0) * t906)) + (static_cast<Real>(-1.0) * t1133)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(t1152), hk::math::abs(t45))))));
            const auto t1160 = (t1159 < static_cast<Real>(1.0));
            const auto t1161 = hk::Item<Real, 6>{t766, t847, t929, t1082, t1117, t1152};
            const auto hz0 = hk::constant<hk::extents<>>(t1160);
            const auto t1166 = (t1160 ? (t4 ? psc_t_end_i : (mut_t_i + t5)) : mut_t_i);
            mut_s[i] = hk::select(hz0, t1161, mut_s_i);
            mut_t[i] = t1166;
            mut_h[i] = (t5 * hk::math::fmin(static_cast<Real>(5.0), hk::math::fmax(static_cast<Real>(0.2), (static_cast<Real>(0.9) * (static_cast<Real>(1.0) / hk::math::sqrt(hk::math::sqrt(hk::math::sqrt(t1159))))))));
            mut_n_acc[i] = (mut_n_acc[i].get()() + (t1160 ? static_cast<Real>(1.0) : static_cast<Real>(0.0)));
            mut_n_rej[i] = (mut_n_rej[i].get()() + (t1160 ? static_cast<Real>(0.0) : static_cast<Real>(1.0)));
            if (!trm_terminated[i].eval() && (t1166 >= psc_t_end_i)) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
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
                const auto mut_s_i = mut_s[i].get();
                const auto mut_t_i = mut_t[i].get()();
                const auto mut_h_i = mut_h[i].get()();
                const auto mut_n_acc_i = mut_n_acc[i].get()();
                const auto mut_n_rej_i = mut_n_rej[i].get()();
                const auto psc_t_end_i = psc_t_end[i].eval();
                const auto t70 = lut_fused_steps[hk::SampleIndex::make(static_cast<std::size_t>(static_cast<Int>(0)))].eval();
                const auto t72 = ((t70 < static_cast<Int>(0)) ? static_cast<Int>(0) : t70);
            hk::Item<Real, 6> hk_c0 = mut_s_i;
            Real hk_c1 = mut_t_i;
            Real hk_c2 = mut_h_i;
            Real hk_c3 = mut_n_acc_i;
            Real hk_c4 = mut_n_rej_i;
            Real hk_c5 = static_cast<Real>(0.0);
            const int hk_cnt = hawk_clamp_count(t72);
            unsigned hk_trip = 0u;
            if (hk_cnt > 0)
            while (true) {
                const int hawk_k73_step = static_cast<int>(hk_trip);
                (void)hawk_k73_step;
                const hk::Item<Real, 6> hawk_v73_0_s = hk_c0;
                const Real hawk_v73_1_t = hk_c1;
                const Real hawk_v73_2_h = hk_c2;
                const Real hawk_v73_3_n_acc = hk_c3;
                const Real hawk_v73_4_n_rej = hk_c4;
                const Real hawk_v73_5_finished = hk_c5;
                    const auto tb0 = (psc_t_end_i - hawk_v73_1_t);
                    const auto tb1 = (hawk_v73_2_h >= tb0);
                    const auto tb2 = (tb1 ? tb0 : hawk_v73_2_h);
                    const auto tb3 = hawk_v73_0_s.eval<3>(i);
                    const auto tb4 = (((hawk_v73_0_s.eval<0>(i) * hawk_v73_0_s.eval<0>(i)) + (hawk_v73_0_s.eval<1>(i) * hawk_v73_0_s.eval<1>(i))) + (hawk_v73_0_s.eval<2>(i) * hawk_v73_0_s.eval<2>(i)));
                    const auto tb5 = (static_cast<Real>(1.0) / (tb4 * hk::math::sqrt(tb4)));
                    const auto tb6 = (-(hawk_v73_0_s.eval<0>(i) * tb5));
                    const auto tb7 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb3)));
                    const auto tb8 = hawk_v73_0_s.eval<4>(i);
                    const auto tb9 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb8)));
                    const auto tb10 = hawk_v73_0_s.eval<5>(i);
                    const auto tb11 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb10)));
                    const auto tb12 = (((tb7 * tb7) + (tb9 * tb9)) + (tb11 * tb11));
                    const auto tb13 = (static_cast<Real>(1.0) / (tb12 * hk::math::sqrt(tb12)));
                    const auto tb14 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb6) + (static_cast<Real>(0.08333333333333333) * (-(tb7 * tb13))))));
                    const auto tb15 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb3) + (static_cast<Real>(0.125) * tb14))));
                    const auto tb16 = (-(hawk_v73_0_s.eval<1>(i) * tb5));
                    const auto tb17 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb16) + (static_cast<Real>(0.08333333333333333) * (-(tb9 * tb13))))));
                    const auto tb18 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb8) + (static_cast<Real>(0.125) * tb17))));
                    const auto tb19 = (-(hawk_v73_0_s.eval<2>(i) * tb5));
                    const auto tb20 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb19) + (static_cast<Real>(0.08333333333333333) * (-(tb11 * tb13))))));
                    const auto tb21 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb10) + (static_cast<Real>(0.125) * tb20))));
                    const auto tb22 = (((tb15 * tb15) + (tb18 * tb18)) + (tb21 * tb21));
                    const auto tb23 = (static_cast<Real>(1.0) / (tb22 * hk::math::sqrt(tb22)));
                    const auto tb24 = (-(tb15 * tb23));
                    const auto tb25 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb3) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<3>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb6)))))));
                    const auto tb26 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb8) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<4>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb16)))))));
                    const auto tb27 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((static_cast<Real>(0.027777777777777776) * tb10) + (static_cast<Real>(0.08333333333333333) * (hawk_v73_0_s.eval<5>(i) + (tb2 * (static_cast<Real>(0.07407407407407407) * tb19)))))));
                    const auto tb28 = (((tb25 * tb25) + (tb26 * tb26)) + (tb27 * tb27));
                    const auto tb29 = (static_cast<Real>(1.0) / (tb28 * hk::math::sqrt(tb28)));
                    const auto tb30 = (-(tb25 * tb29));
                    const auto tb31 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb6) + (static_cast<Real>(0.125) * tb30))));
                    const auto tb32 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb3) + (static_cast<Real>(-1.5625) * tb14)) + (static_cast<Real>(1.5625) * tb31))));
                    const auto tb33 = (-(tb26 * tb29));
                    const auto tb34 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb16) + (static_cast<Real>(0.125) * tb33))));
                    const auto tb35 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb8) + (static_cast<Real>(-1.5625) * tb17)) + (static_cast<Real>(1.5625) * tb34))));
                    const auto tb36 = (-(tb27 * tb29));
                    const auto tb37 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((static_cast<Real>(0.041666666666666664) * tb19) + (static_cast<Real>(0.125) * tb36))));
                    const auto tb38 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb10) + (static_cast<Real>(-1.5625) * tb20)) + (static_cast<Real>(1.5625) * tb37))));
                    const auto tb39 = (((tb32 * tb32) + (tb35 * tb35)) + (tb38 * tb38));
                    const auto tb40 = (static_cast<Real>(1.0) / (tb39 * hk::math::sqrt(tb39)));
                    const auto tb41 = (-(tb32 * tb40));
                    const auto tb42 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb6) + (static_cast<Real>(-1.5625) * tb30)) + (static_cast<Real>(1.5625) * tb24))));
                    const auto tb43 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((static_cast<Real>(0.05) * tb3) + (static_cast<Real>(0.25) * tb31)) + (static_cast<Real>(0.2) * tb42))));
                    const auto tb44 = (-(tb18 * tb23));
                    const auto tb45 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb16) + (static_cast<Real>(-1.5625) * tb33)) + (static_cast<Real>(1.5625) * tb44))));
                    const auto tb46 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((static_cast<Real>(0.05) * tb8) + (static_cast<Real>(0.25) * tb34)) + (static_cast<Real>(0.2) * tb45))));
                    const auto tb47 = (-(tb21 * tb23));
                    const auto tb48 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((static_cast<Real>(0.4166666666666667) * tb19) + (static_cast<Real>(-1.5625) * tb36)) + (static_cast<Real>(1.5625) * tb47))));
                    const auto tb49 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((static_cast<Real>(0.05) * tb10) + (static_cast<Real>(0.25) * tb37)) + (static_cast<Real>(0.2) * tb48))));
                    const auto tb50 = (((tb43 * tb43) + (tb46 * tb46)) + (tb49 * tb49));
                    const auto tb51 = (static_cast<Real>(1.0) / (tb50 * hk::math::sqrt(tb50)));
                    const auto tb52 = (-(tb43 * tb51));
                    const auto tb53 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((static_cast<Real>(0.05) * tb6) + (static_cast<Real>(0.25) * tb24)) + (static_cast<Real>(0.2) * tb41))));
                    const auto tb54 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb3) + (static_cast<Real>(1.1574074074074074) * tb31)) + (static_cast<Real>(-2.4074074074074074) * tb42)) + (static_cast<Real>(2.314814814814815) * tb53))));
                    const auto tb55 = (-(tb35 * tb40));
                    const auto tb56 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((static_cast<Real>(0.05) * tb16) + (static_cast<Real>(0.25) * tb44)) + (static_cast<Real>(0.2) * tb55))));
                    const auto tb57 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb8) + (static_cast<Real>(1.1574074074074074) * tb34)) + (static_cast<Real>(-2.4074074074074074) * tb45)) + (static_cast<Real>(2.314814814814815) * tb56))));
                    const auto tb58 = (-(tb38 * tb40));
                    const auto tb59 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((static_cast<Real>(0.05) * tb19) + (static_cast<Real>(0.25) * tb47)) + (static_cast<Real>(0.2) * tb58))));
                    const auto tb60 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb10) + (static_cast<Real>(1.1574074074074074) * tb37)) + (static_cast<Real>(-2.4074074074074074) * tb48)) + (static_cast<Real>(2.314814814814815) * tb59))));
                    const auto tb61 = (((tb54 * tb54) + (tb57 * tb57)) + (tb60 * tb60));
                    const auto tb62 = (static_cast<Real>(1.0) / (tb61 * hk::math::sqrt(tb61)));
                    const auto tb63 = (-(tb54 * tb62));
                    const auto tb64 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb6) + (static_cast<Real>(1.1574074074074074) * tb24)) + (static_cast<Real>(-2.4074074074074074) * tb41)) + (static_cast<Real>(2.314814814814815) * tb52))));
                    const auto tb65 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb3) + (static_cast<Real>(0.27111111111111114) * tb42)) + (static_cast<Real>(-0.2222222222222222) * tb53)) + (static_cast<Real>(0.014444444444444444) * tb64))));
                    const auto tb66 = (-(tb46 * tb51));
                    const auto tb67 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb16) + (static_cast<Real>(1.1574074074074074) * tb44)) + (static_cast<Real>(-2.4074074074074074) * tb55)) + (static_cast<Real>(2.314814814814815) * tb66))));
                    const auto tb68 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb8) + (static_cast<Real>(0.27111111111111114) * tb45)) + (static_cast<Real>(-0.2222222222222222) * tb56)) + (static_cast<Real>(0.014444444444444444) * tb67))));
                    const auto tb69 = (-(tb49 * tb51));
                    const auto tb70 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((static_cast<Real>(-0.23148148148148148) * tb19) + (static_cast<Real>(1.1574074074074074) * tb47)) + (static_cast<Real>(-2.4074074074074074) * tb58)) + (static_cast<Real>(2.314814814814815) * tb69))));
                    const auto tb71 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb10) + (static_cast<Real>(0.27111111111111114) * tb48)) + (static_cast<Real>(-0.2222222222222222) * tb59)) + (static_cast<Real>(0.014444444444444444) * tb70))));
                    const auto tb72 = (((tb65 * tb65) + (tb68 * tb68)) + (tb71 * tb71));
                    const auto tb73 = (static_cast<Real>(1.0) / (tb72 * hk::math::sqrt(tb72)));
                    const auto tb74 = (-(tb65 * tb73));
                    const auto tb75 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb6) + (static_cast<Real>(0.27111111111111114) * tb41)) + (static_cast<Real>(-0.2222222222222222) * tb52)) + (static_cast<Real>(0.014444444444444444) * tb63))));
                    const auto tb76 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb3) + (static_cast<Real>(-8.833333333333334) * tb31)) + (static_cast<Real>(15.644444444444444) * tb42)) + (static_cast<Real>(-11.88888888888889) * tb53)) + (static_cast<Real>(0.7444444444444445) * tb64)) + (static_cast<Real>(3.0) * tb75))));
                    const auto tb77 = (-(tb57 * tb62));
                    const auto tb78 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb16) + (static_cast<Real>(0.27111111111111114) * tb55)) + (static_cast<Real>(-0.2222222222222222) * tb66)) + (static_cast<Real>(0.014444444444444444) * tb77))));
                    const auto tb79 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb8) + (static_cast<Real>(-8.833333333333334) * tb34)) + (static_cast<Real>(15.644444444444444) * tb45)) + (static_cast<Real>(-11.88888888888889) * tb56)) + (static_cast<Real>(0.7444444444444445) * tb67)) + (static_cast<Real>(3.0) * tb78))));
                    const auto tb80 = (-(tb60 * tb62));
                    const auto tb81 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((static_cast<Real>(0.10333333333333333) * tb19) + (static_cast<Real>(0.27111111111111114) * tb58)) + (static_cast<Real>(-0.2222222222222222) * tb69)) + (static_cast<Real>(0.014444444444444444) * tb80))));
                    const auto tb82 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb10) + (static_cast<Real>(-8.833333333333334) * tb37)) + (static_cast<Real>(15.644444444444444) * tb48)) + (static_cast<Real>(-11.88888888888889) * tb59)) + (static_cast<Real>(0.7444444444444445) * tb70)) + (static_cast<Real>(3.0) * tb81))));
                    const auto tb83 = (((tb76 * tb76) + (tb79 * tb79)) + (tb82 * tb82));
                    const auto tb84 = (static_cast<Real>(1.0) / (tb83 * hk::math::sqrt(tb83)));
                    const auto tb85 = (-(tb76 * tb84));
                    const auto tb86 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb6) + (static_cast<Real>(-8.833333333333334) * tb24)) + (static_cast<Real>(15.644444444444444) * tb41)) + (static_cast<Real>(-11.88888888888889) * tb52)) + (static_cast<Real>(0.7444444444444445) * tb63)) + (static_cast<Real>(3.0) * tb74))));
                    const auto tb87 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb3) + (static_cast<Real>(0.21296296296296297) * tb31)) + (static_cast<Real>(-7.229629629629629) * tb42)) + (static_cast<Real>(5.7592592592592595) * tb53)) + (static_cast<Real>(-0.31666666666666665) * tb64)) + (static_cast<Real>(2.8333333333333335) * tb75)) + (static_cast<Real>(-0.08333333333333333) * tb86))));
                    const auto tb88 = (-(tb68 * tb73));
                    const auto tb89 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb16) + (static_cast<Real>(-8.833333333333334) * tb44)) + (static_cast<Real>(15.644444444444444) * tb55)) + (static_cast<Real>(-11.88888888888889) * tb66)) + (static_cast<Real>(0.7444444444444445) * tb77)) + (static_cast<Real>(3.0) * tb88))));
                    const auto tb90 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb8) + (static_cast<Real>(0.21296296296296297) * tb34)) + (static_cast<Real>(-7.229629629629629) * tb45)) + (static_cast<Real>(5.7592592592592595) * tb56)) + (static_cast<Real>(-0.31666666666666665) * tb67)) + (static_cast<Real>(2.8333333333333335) * tb78)) + (static_cast<Real>(-0.08333333333333333) * tb89))));
                    const auto tb91 = (-(tb71 * tb73));
                    const auto tb92 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((static_cast<Real>(2.0) * tb19) + (static_cast<Real>(-8.833333333333334) * tb47)) + (static_cast<Real>(15.644444444444444) * tb58)) + (static_cast<Real>(-11.88888888888889) * tb69)) + (static_cast<Real>(0.7444444444444445) * tb80)) + (static_cast<Real>(3.0) * tb91))));
                    const auto tb93 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb10) + (static_cast<Real>(0.21296296296296297) * tb37)) + (static_cast<Real>(-7.229629629629629) * tb48)) + (static_cast<Real>(5.7592592592592595) * tb59)) + (static_cast<Real>(-0.31666666666666665) * tb70)) + (static_cast<Real>(2.8333333333333335) * tb81)) + (static_cast<Real>(-0.08333333333333333) * tb92))));
                    const auto tb94 = (((tb87 * tb87) + (tb90 * tb90)) + (tb93 * tb93));
                    const auto tb95 = (static_cast<Real>(1.0) / (tb94 * hk::math::sqrt(tb94)));
                    const auto tb96 = (-(tb87 * tb95));
                    const auto tb97 = (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb6) + (static_cast<Real>(-0.14634146341463414) * tb52)) + (static_cast<Real>(-0.014634146341463415) * tb63)) + (static_cast<Real>(-0.07317073170731707) * tb74)) + (static_cast<Real>(0.07317073170731707) * tb85)) + (static_cast<Real>(0.14634146341463414) * tb96))));
                    const auto tb98 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb6) + (static_cast<Real>(0.21296296296296297) * tb24)) + (static_cast<Real>(-7.229629629629629) * tb41)) + (static_cast<Real>(5.7592592592592595) * tb52)) + (static_cast<Real>(-0.31666666666666665) * tb63)) + (static_cast<Real>(2.8333333333333335) * tb74)) + (static_cast<Real>(-0.08333333333333333) * tb85))));
                    const auto tb99 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb3) + (static_cast<Real>(-0.14634146341463414) * tb53)) + (static_cast<Real>(-0.014634146341463415) * tb64)) + (static_cast<Real>(-0.07317073170731707) * tb75)) + (static_cast<Real>(0.07317073170731707) * tb86)) + (static_cast<Real>(0.14634146341463414) * tb98))));
                    const auto tb100 = (-(tb79 * tb84));
                    const auto tb101 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb16) + (static_cast<Real>(0.21296296296296297) * tb44)) + (static_cast<Real>(-7.229629629629629) * tb55)) + (static_cast<Real>(5.7592592592592595) * tb66)) + (static_cast<Real>(-0.31666666666666665) * tb77)) + (static_cast<Real>(2.8333333333333335) * tb88)) + (static_cast<Real>(-0.08333333333333333) * tb100))));
                    const auto tb102 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb8) + (static_cast<Real>(-0.14634146341463414) * tb56)) + (static_cast<Real>(-0.014634146341463415) * tb67)) + (static_cast<Real>(-0.07317073170731707) * tb78)) + (static_cast<Real>(0.07317073170731707) * tb89)) + (static_cast<Real>(0.14634146341463414) * tb101))));
                    const auto tb103 = (-(tb82 * tb84));
                    const auto tb104 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((static_cast<Real>(-0.8425925925925926) * tb19) + (static_cast<Real>(0.21296296296296297) * tb47)) + (static_cast<Real>(-7.229629629629629) * tb58)) + (static_cast<Real>(5.7592592592592595) * tb69)) + (static_cast<Real>(-0.31666666666666665) * tb80)) + (static_cast<Real>(2.8333333333333335) * tb91)) + (static_cast<Real>(-0.08333333333333333) * tb103))));
                    const auto tb105 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb10) + (static_cast<Real>(-0.14634146341463414) * tb59)) + (static_cast<Real>(-0.014634146341463415) * tb70)) + (static_cast<Real>(-0.07317073170731707) * tb81)) + (static_cast<Real>(0.07317073170731707) * tb92)) + (static_cast<Real>(0.14634146341463414) * tb104))));
                    const auto tb106 = (((tb99 * tb99) + (tb102 * tb102)) + (tb105 * tb105));
                    const auto tb107 = (static_cast<Real>(1.0) / (tb106 * hk::math::sqrt(tb106)));
                    const auto tb108 = (-(tb99 * tb107));
                    const auto tb109 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb6) + (static_cast<Real>(-2.0792682926829267) * tb24)) + (static_cast<Real>(4.3863414634146345) * tb41)) + (static_cast<Real>(-3.524390243902439) * tb52)) + (static_cast<Real>(0.5348780487804878) * tb63)) + (static_cast<Real>(0.6219512195121951) * tb74)) + (static_cast<Real>(0.20121951219512196) * tb85)) + (static_cast<Real>(0.2926829268292683) * tb96)) + (static_cast<Real>(1.0) * tb108))));
                    const auto tb110 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb53) + (static_cast<Real>(0.2571428571428571) * tb64)) + (static_cast<Real>(0.2571428571428571) * tb75)) + (static_cast<Real>(0.03214285714285714) * tb86)) + (static_cast<Real>(0.03214285714285714) * tb98)) + (static_cast<Real>(0.04880952380952381) * tb97)) + (static_cast<Real>(0.04880952380952381) * tb109))));
                    const auto tb111 = (-(tb90 * tb95));
                    const auto tb112 = (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb16) + (static_cast<Real>(-0.14634146341463414) * tb66)) + (static_cast<Real>(-0.014634146341463415) * tb77)) + (static_cast<Real>(-0.07317073170731707) * tb88)) + (static_cast<Real>(0.07317073170731707) * tb100)) + (static_cast<Real>(0.14634146341463414) * tb111))));
                    const auto tb113 = (-(tb102 * tb107));
                    const auto tb114 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb16) + (static_cast<Real>(-2.0792682926829267) * tb44)) + (static_cast<Real>(4.3863414634146345) * tb55)) + (static_cast<Real>(-3.524390243902439) * tb66)) + (static_cast<Real>(0.5348780487804878) * tb77)) + (static_cast<Real>(0.6219512195121951) * tb88)) + (static_cast<Real>(0.20121951219512196) * tb100)) + (static_cast<Real>(0.2926829268292683) * tb111)) + (static_cast<Real>(1.0) * tb113))));
                    const auto tb115 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb56) + (static_cast<Real>(0.2571428571428571) * tb67)) + (static_cast<Real>(0.2571428571428571) * tb78)) + (static_cast<Real>(0.03214285714285714) * tb89)) + (static_cast<Real>(0.03214285714285714) * tb101)) + (static_cast<Real>(0.04880952380952381) * tb112)) + (static_cast<Real>(0.04880952380952381) * tb114))));
                    const auto tb116 = (-(tb93 * tb95));
                    const auto tb117 = (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((static_cast<Real>(0.014634146341463415) * tb19) + (static_cast<Real>(-0.14634146341463414) * tb69)) + (static_cast<Real>(-0.014634146341463415) * tb80)) + (static_cast<Real>(-0.07317073170731707) * tb91)) + (static_cast<Real>(0.07317073170731707) * tb103)) + (static_cast<Real>(0.14634146341463414) * tb116))));
                    const auto tb118 = (-(tb105 * tb107));
                    const auto tb119 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb19) + (static_cast<Real>(-2.0792682926829267) * tb47)) + (static_cast<Real>(4.3863414634146345) * tb58)) + (static_cast<Real>(-3.524390243902439) * tb69)) + (static_cast<Real>(0.5348780487804878) * tb80)) + (static_cast<Real>(0.6219512195121951) * tb91)) + (static_cast<Real>(0.20121951219512196) * tb103)) + (static_cast<Real>(0.2926829268292683) * tb116)) + (static_cast<Real>(1.0) * tb118))));
                    const auto tb120 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb59) + (static_cast<Real>(0.2571428571428571) * tb70)) + (static_cast<Real>(0.2571428571428571) * tb81)) + (static_cast<Real>(0.03214285714285714) * tb92)) + (static_cast<Real>(0.03214285714285714) * tb104)) + (static_cast<Real>(0.04880952380952381) * tb117)) + (static_cast<Real>(0.04880952380952381) * tb119))));
                    const auto tb121 = (hawk_v73_0_s.eval<0>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb3) + (static_cast<Real>(-2.0792682926829267) * tb31)) + (static_cast<Real>(4.3863414634146345) * tb42)) + (static_cast<Real>(-3.6707317073170733) * tb53)) + (static_cast<Real>(0.5202439024390244) * tb64)) + (static_cast<Real>(0.5487804878048781) * tb75)) + (static_cast<Real>(0.27439024390243905) * tb86)) + (static_cast<Real>(0.43902439024390244) * tb98))));
                    const auto tb122 = (hawk_v73_0_s.eval<1>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb8) + (static_cast<Real>(-2.0792682926829267) * tb34)) + (static_cast<Real>(4.3863414634146345) * tb45)) + (static_cast<Real>(-3.6707317073170733) * tb56)) + (static_cast<Real>(0.5202439024390244) * tb67)) + (static_cast<Real>(0.5487804878048781) * tb78)) + (static_cast<Real>(0.27439024390243905) * tb89)) + (static_cast<Real>(0.43902439024390244) * tb101))));
                    const auto tb123 = (hawk_v73_0_s.eval<2>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb10) + (static_cast<Real>(-2.0792682926829267) * tb37)) + (static_cast<Real>(4.3863414634146345) * tb48)) + (static_cast<Real>(-3.6707317073170733) * tb59)) + (static_cast<Real>(0.5202439024390244) * tb70)) + (static_cast<Real>(0.5487804878048781) * tb81)) + (static_cast<Real>(0.27439024390243905) * tb92)) + (static_cast<Real>(0.43902439024390244) * tb104))));
                    const auto tb124 = (((tb121 * tb121) + (tb122 * tb122)) + (tb123 * tb123));
                    const auto tb125 = (static_cast<Real>(1.0) / (tb124 * hk::math::sqrt(tb124)));
                    const auto tb126 = (hawk_v73_0_s.eval<0>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb3) + (static_cast<Real>(-2.0792682926829267) * tb31)) + (static_cast<Real>(4.3863414634146345) * tb42)) + (static_cast<Real>(-3.524390243902439) * tb53)) + (static_cast<Real>(0.5348780487804878) * tb64)) + (static_cast<Real>(0.6219512195121951) * tb75)) + (static_cast<Real>(0.20121951219512196) * tb86)) + (static_cast<Real>(0.2926829268292683) * tb98)) + (static_cast<Real>(1.0) * tb97))));
                    const auto tb127 = (hawk_v73_0_s.eval<1>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb8) + (static_cast<Real>(-2.0792682926829267) * tb34)) + (static_cast<Real>(4.3863414634146345) * tb45)) + (static_cast<Real>(-3.524390243902439) * tb56)) + (static_cast<Real>(0.5348780487804878) * tb67)) + (static_cast<Real>(0.6219512195121951) * tb78)) + (static_cast<Real>(0.20121951219512196) * tb89)) + (static_cast<Real>(0.2926829268292683) * tb101)) + (static_cast<Real>(1.0) * tb112))));
                    const auto tb128 = (hawk_v73_0_s.eval<2>(i) + (tb2 * (((((((((static_cast<Real>(-0.43341463414634146) * tb10) + (static_cast<Real>(-2.0792682926829267) * tb37)) + (static_cast<Real>(4.3863414634146345) * tb48)) + (static_cast<Real>(-3.524390243902439) * tb59)) + (static_cast<Real>(0.5348780487804878) * tb70)) + (static_cast<Real>(0.6219512195121951) * tb81)) + (static_cast<Real>(0.20121951219512196) * tb92)) + (static_cast<Real>(0.2926829268292683) * tb104)) + (static_cast<Real>(1.0) * tb117))));
                    const auto tb129 = (((tb126 * tb126) + (tb127 * tb127)) + (tb128 * tb128));
                    const auto tb130 = (static_cast<Real>(1.0) / (tb129 * hk::math::sqrt(tb129)));
                    const auto tb131 = (-(tb126 * tb130));
                    const auto tb132 = (hawk_v73_0_s.eval<3>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb52) + (static_cast<Real>(0.2571428571428571) * tb63)) + (static_cast<Real>(0.2571428571428571) * tb74)) + (static_cast<Real>(0.03214285714285714) * tb85)) + (static_cast<Real>(0.03214285714285714) * tb96)) + (static_cast<Real>(0.04880952380952381) * tb108)) + (static_cast<Real>(0.04880952380952381) * tb131))));
                    const auto tb133 = (-(tb127 * tb130));
                    const auto tb134 = (hawk_v73_0_s.eval<4>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb66) + (static_cast<Real>(0.2571428571428571) * tb77)) + (static_cast<Real>(0.2571428571428571) * tb88)) + (static_cast<Real>(0.03214285714285714) * tb100)) + (static_cast<Real>(0.03214285714285714) * tb111)) + (static_cast<Real>(0.04880952380952381) * tb113)) + (static_cast<Real>(0.04880952380952381) * tb133))));
                    const auto tb135 = (-(tb128 * tb130));
                    const auto tb136 = (hawk_v73_0_s.eval<5>(i) + (tb2 * (((((((static_cast<Real>(0.3238095238095238) * tb69) + (static_cast<Real>(0.2571428571428571) * tb80)) + (static_cast<Real>(0.2571428571428571) * tb91)) + (static_cast<Real>(0.03214285714285714) * tb103)) + (static_cast<Real>(0.03214285714285714) * tb116)) + (static_cast<Real>(0.04880952380952381) * tb118)) + (static_cast<Real>(0.04880952380952381) * tb135))));
                    const auto tb137 = hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax(hk::math::fmax((hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb3) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<3>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb6) + (static_cast<Real>(-2.0792682926829267) * tb24)) + (static_cast<Real>(4.3863414634146345) * tb41)) + (static_cast<Real>(-3.6707317073170733) * tb52)) + (static_cast<Real>(0.5202439024390244) * tb63)) + (static_cast<Real>(0.5487804878048781) * tb74)) + (static_cast<Real>(0.27439024390243905) * tb85)) + (static_cast<Real>(0.43902439024390244) * tb96)))))) + (static_cast<Real>(-1.0) * tb97)) + (static_cast<Real>(-1.0) * tb109)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb110), hk::math::abs(hawk_v73_0_s.eval<0>(i)))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb8) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<4>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb16) + (static_cast<Real>(-2.0792682926829267) * tb44)) + (static_cast<Real>(4.3863414634146345) * tb55)) + (static_cast<Real>(-3.6707317073170733) * tb66)) + (static_cast<Real>(0.5202439024390244) * tb77)) + (static_cast<Real>(0.5487804878048781) * tb88)) + (static_cast<Real>(0.27439024390243905) * tb100)) + (static_cast<Real>(0.43902439024390244) * tb111)))))) + (static_cast<Real>(-1.0) * tb112)) + (static_cast<Real>(-1.0) * tb114)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb115), hk::math::abs(hawk_v73_0_s.eval<1>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb10) + (static_cast<Real>(1.0) * (hawk_v73_0_s.eval<5>(i) + (tb2 * ((((((((static_cast<Real>(0.5812195121951219) * tb19) + (static_cast<Real>(-2.0792682926829267) * tb47)) + (static_cast<Real>(4.3863414634146345) * tb58)) + (static_cast<Real>(-3.6707317073170733) * tb69)) + (static_cast<Real>(0.5202439024390244) * tb80)) + (static_cast<Real>(0.5487804878048781) * tb91)) + (static_cast<Real>(0.27439024390243905) * tb103)) + (static_cast<Real>(0.43902439024390244) * tb116)))))) + (static_cast<Real>(-1.0) * tb117)) + (static_cast<Real>(-1.0) * tb119)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb120), hk::math::abs(hawk_v73_0_s.eval<2>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb6) + (static_cast<Real>(1.0) * (-(tb121 * tb125)))) + (static_cast<Real>(-1.0) * tb108)) + (static_cast<Real>(-1.0) * tb131)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb132), hk::math::abs(hawk_v73_0_s.eval<3>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb16) + (static_cast<Real>(1.0) * (-(tb122 * tb125)))) + (static_cast<Real>(-1.0) * tb113)) + (static_cast<Real>(-1.0) * tb133)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb134), hk::math::abs(hawk_v73_0_s.eval<4>(i))))))), (hk::math::abs(((tb2 * static_cast<Real>(0.04880952380952381)) * ((((static_cast<Real>(1.0) * tb19) + (static_cast<Real>(1.0) * (-(tb123 * tb125)))) + (static_cast<Real>(-1.0) * tb118)) + (static_cast<Real>(-1.0) * tb135)))) / (static_cast<Real>(1e-10) + (static_cast<Real>(1e-10) * hk::math::fmax(hk::math::abs(tb136), hk::math::abs(hawk_v73_0_s.eval<5>(i)))))));
                    const auto tb138 = (tb137 < static_cast<Real>(1.0));
                    const auto tb139 = hk::Item<Real, 6>{tb110, tb115, tb120, tb132, tb134, tb136};
                    const auto hz0 = hk::constant<hk::extents<>>(tb138);
                    const auto tb140 = (tb1 ? psc_t_end_i : (hawk_v73_1_t + tb2));
                    const auto tb141 = (tb138 ? tb140 : hawk_v73_1_t);
                    const auto tb142 = hk::math::fmin(static_cast<Real>(5.0), hk::math::fmax(static_cast<Real>(0.2), (static_cast<Real>(0.9) * (static_cast<Real>(1.0) / hk::math::sqrt(hk::math::sqrt(hk::math::sqrt(tb137)))))));
                    const auto tb143 = (tb138 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                    const auto tb144 = (tb138 ? static_cast<Real>(0.0) : static_cast<Real>(1.0));
                    const auto tb145 = (tb141 >= psc_t_end_i);
                    const hk::Item<Real, 6> hawk_n73_0 = hk::select(hz0, tb139, hawk_v73_0_s);
                    const Real hawk_n73_1 = tb141;
                    const Real hawk_n73_2 = (tb2 * tb142);
                    const Real hawk_n73_3 = (hawk_v73_3_n_acc + tb143);
                    const Real hawk_n73_4 = (hawk_v73_4_n_rej + tb144);
                    const Real hawk_n73_5 = (tb145 ? static_cast<Real>(1.0) : static_cast<Real>(0.0));
                    const bool hawk_x73 = tb145;
                hk_c0 = hawk_n73_0;
                hk_c1 = hawk_n73_1;
                hk_c2 = hawk_n73_2;
                hk_c3 = hawk_n73_3;
                hk_c4 = hawk_n73_4;
                hk_c5 = hawk_n73_5;
                ++hk_trip;
                if (hawk_x73 || hk_trip >= static_cast<unsigned>(hk_cnt)) break;
            }
            {
                const hk::Item<Real, 6> hawk_v73_0_s = hk_c0;
                const Real hawk_v73_1_t = hk_c1;
                const Real hawk_v73_2_h = hk_c2;
                const Real hawk_v73_3_n_acc = hk_c3;
                const Real hawk_v73_4_n_rej = hk_c4;
                const Real hawk_v73_5_finished = hk_c5;
                (void)hawk_v73_0_s;
                (void)hawk_v73_1_t;
                (void)hawk_v73_2_h;
                (void)hawk_v73_3_n_acc;
                (void)hawk_v73_4_n_rej;
                (void)hawk_v73_5_finished;
                mut_s[i] = hawk_v73_0_s;
                mut_t[i] = hawk_v73_1_t;
                mut_h[i] = hawk_v73_2_h;
                mut_n_acc[i] = hawk_v73_3_n_acc;
                mut_n_rej[i] = hawk_v73_4_n_rej;
                if (!trm_terminated[i].eval() && (hawk_v73_5_finished > static_cast<Real>(0.5))) { trm_terminated_w[i] = true; hawk_abi::finish_count(lut_finished_count); }
            }
            hk_longest = hk_trip > hk_longest ? hk_trip : hk_longest;
            hk_ran += hk_trip;
        } else { hawk_abi::finish_count(lut_finished_count); }
    }
    }
    // one report per warp: the longest trip count and the steps run
    hk::persist_report(hawk_steps, hawk_stepsum, nullptr, hk_longest, hk_ran);
}
