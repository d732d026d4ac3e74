// hawk_b200 unit 'spd_solve_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(128, 5) spd_solve_vjp(
    hk::abi::GRefMirror p_mut_bar_A,
    hk::abi::GRefMirror p_mut_bar_b,
    hk::abi::GRefMirror p_vin_b,
    hk::abi::GRefMirror p_vin_bar_x,
    hk::abi::GRefMirror p_mtx_A,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::MatOut<Real, 6, 6> mut_bar_A(p_mut_bar_A);
    (void)mut_bar_A;
    const hk::VecOut<Real, 6> mut_bar_b(p_mut_bar_b);
    (void)mut_bar_b;
    const hk::VecIn<Real, 6> vin_b(p_vin_b);
    (void)vin_b;
    const hk::VecIn<Real, 6> vin_bar_x(p_vin_bar_x);
    (void)vin_bar_x;
    const hk::MatIn<Real, 6, 6> mtx_A(p_mtx_A);
    (void)mtx_A;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto mtx_A_i = mtx_A[i].get();
        hk::linalg::Cholesky<Real, 6> hawk_lf0;
        hk::linalg::cholesky<6>(hawk_lf0, mtx_A[i]);
        const auto t1 = hawk_lf0;
        const auto vin_bar_x_i = vin_bar_x[i].get();
        hk::Item<Real, 6> hawk_la1;
        hk::linalg::choSolve<1>(t1, vin_bar_x[i], hawk_la1);
        const hk::Item<Real, 6> t3 = hawk_la1;
        mut_bar_b[i] = t3;
        const auto vin_b_i = vin_b[i].get();
        hk::Item<Real, 6> hawk_la2;
        hk::linalg::choSolve<1>(t1, vin_b[i], hawk_la2);
        const auto t6 = hk::outer(t3, hawk_la2);
        mut_bar_A[i] = (((t6 + t6.transpose()) * static_cast<Real>(0.5)) * static_cast<Real>(-1));
    }
}
