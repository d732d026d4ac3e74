// hawk_b200 unit 'sym_eigen' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS

extern "C" __global__ void __launch_bounds__(256) sym_eigen(
    hk::abi::GRefMirror p_mut_V,
    hk::abi::ScalarHandle p_mut_info,
    hk::abi::GRefMirror p_mut_w,
    hk::abi::GRefMirror p_mtx_A,
    long long base,
    long long count,
    long long nSamples)
{
    const hk::MatOut<Real, 6, 6> mut_V(p_mut_V);
    (void)mut_V;
    const hk::ScalarOut<std::int32_t> mut_info(p_mut_info);
    (void)mut_info;
    const hk::VecOut<Real, 6> mut_w(p_mut_w);
    (void)mut_w;
    const hk::MatIn<Real, 6, 6> mtx_A(p_mtx_A);
    (void)mtx_A;
    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; hawk_flat += hk::lane_step()) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i};
        (void)hawk_i;
        (void)nSamples;
        const auto mtx_A_i = mtx_A[i].get();
        hk::linalg::Eigh<Real, 6> hawk_lf0;
        hk::linalg::eigh<6>(hawk_lf0, mtx_A[i]);
        const auto t1 = hawk_lf0;
        hk::Item<Real, 6> hawk_la1;
        for (Int hawk_lk = 0; hawk_lk < 6; ++hawk_lk) hawk_la1.data()[hawk_lk] = t1.w[hawk_lk];
        mut_w[i] = hawk_la1;
        hk::Item<Real, 6, 6> hawk_la2;
        for (Int hawk_lk = 0; hawk_lk < 36; ++hawk_lk) hawk_la2.data()[hawk_lk] = t1.v[hawk_lk];
        mut_V[i] = hawk_la2;
        mut_info[i] = t1.info;
    }
}
