// hawk_b200 unit 'spd_solve_vjp' (scalar mode float64), sm_100a.
// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.
#include "hk/hawk_b200.cuh"

using Real = double;
using Int = long long;

HK_SELF_CHECK_EXPORTS
HK_DYNAMIC_SMEM(196736)

extern "C" __global__ void __launch_bounds__(256) spd_solve_vjp(
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
    const hk::VecIn<Real, 6> vin_b(p_vin_b, 0u, 2048u);
    (void)vin_b;
    const hk::VecIn<Real, 6> vin_bar_x(p_vin_bar_x, 12288u, 2048u);
    (void)vin_bar_x;
    const hk::MatIn<Real, 6, 6> mtx_A(p_mtx_A, 24576u, 2048u);
    (void)mtx_A;
    extern __shared__ __align__(128) unsigned char hk_smem[];
    hk::stage::Pipe<2> hk_pipe(hk_smem, 98304u, 98304u);
    const bool hk_aligned = hk::stage::aligned(vin_b.data(), vin_b.pitch * sizeof(*vin_b.data()), base * static_cast<long long>(sizeof(*vin_b.data()))) && hk::stage::aligned(vin_bar_x.data(), vin_bar_x.pitch * sizeof(*vin_bar_x.data()), base * static_cast<long long>(sizeof(*vin_bar_x.data()))) && hk::stage::aligned(mtx_A.data(), mtx_A.pitch * sizeof(*mtx_A.data()), base * static_cast<long long>(sizeof(*mtx_A.data())));
    const long long hk_tiles = (count + 255) >> 8;
    const long long hk_mine = hk_tiles > static_cast<long long>(blockIdx.x) ? (hk_tiles - 1 - static_cast<long long>(blockIdx.x)) / gridDim.x + 1 : 0;
    const long long hk_full = count >> 8;
    const long long hk_staged = (!hk_aligned || hk_full <= static_cast<long long>(blockIdx.x)) ? 0 : (hk_full - 1 - static_cast<long long>(blockIdx.x)) / gridDim.x + 1;
    auto hk_issue = [&](long long hk_jj, unsigned char* hk_to, unsigned long long* hk_bar) {
        const long long hk_first = (static_cast<long long>(blockIdx.x) + hk_jj * gridDim.x) << 8;
        hk::stage::copy(hk_to + 0u, vin_b.data() + 0ull * vin_b.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 2048u, vin_b.data() + 1ull * vin_b.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 4096u, vin_b.data() + 2ull * vin_b.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 6144u, vin_b.data() + 3ull * vin_b.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 8192u, vin_b.data() + 4ull * vin_b.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 10240u, vin_b.data() + 5ull * vin_b.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 12288u, vin_bar_x.data() + 0ull * vin_bar_x.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 14336u, vin_bar_x.data() + 1ull * vin_bar_x.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 16384u, vin_bar_x.data() + 2ull * vin_bar_x.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 18432u, vin_bar_x.data() + 3ull * vin_bar_x.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 20480u, vin_bar_x.data() + 4ull * vin_bar_x.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 22528u, vin_bar_x.data() + 5ull * vin_bar_x.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 24576u, mtx_A.data() + 0ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 26624u, mtx_A.data() + 1ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 28672u, mtx_A.data() + 2ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 30720u, mtx_A.data() + 3ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 32768u, mtx_A.data() + 4ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 34816u, mtx_A.data() + 5ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 36864u, mtx_A.data() + 6ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 38912u, mtx_A.data() + 7ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 40960u, mtx_A.data() + 8ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 43008u, mtx_A.data() + 9ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 45056u, mtx_A.data() + 10ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 47104u, mtx_A.data() + 11ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 49152u, mtx_A.data() + 12ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 51200u, mtx_A.data() + 13ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 53248u, mtx_A.data() + 14ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 55296u, mtx_A.data() + 15ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 57344u, mtx_A.data() + 16ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 59392u, mtx_A.data() + 17ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 61440u, mtx_A.data() + 18ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 63488u, mtx_A.data() + 19ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 65536u, mtx_A.data() + 20ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 67584u, mtx_A.data() + 21ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 69632u, mtx_A.data() + 22ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 71680u, mtx_A.data() + 23ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 73728u, mtx_A.data() + 24ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 75776u, mtx_A.data() + 25ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 77824u, mtx_A.data() + 26ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 79872u, mtx_A.data() + 27ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 81920u, mtx_A.data() + 28ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 83968u, mtx_A.data() + 29ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 86016u, mtx_A.data() + 30ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 88064u, mtx_A.data() + 31ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 90112u, mtx_A.data() + 32ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 92160u, mtx_A.data() + 33ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 94208u, mtx_A.data() + 34ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
        hk::stage::copy(hk_to + 96256u, mtx_A.data() + 35ull * mtx_A.pitch + base + hk_first, 2048u, hk_bar);
    };
    hk_pipe.setup(8u);
    bool hk_ok = true;
    if (threadIdx.x == 0)
        for (long long hk_jj = 0; hk_jj < 2 && hk_jj < hk_staged && hk_ok; ++hk_jj)
            hk_ok = hk_pipe.fill(hk_jj, [&](unsigned char* a, unsigned long long* b) { hk_issue(hk_jj, a, b); });
    hk_ok = __shfl_sync(0xffffffffu, hk_ok, 0);
    for (long long hk_j = 0; hk_j < hk_mine && hk_ok; ++hk_j) {
        const long long hk_t = static_cast<long long>(blockIdx.x) + hk_j * gridDim.x;
        const bool hk_use = hk_j < hk_staged;
        const unsigned char* hk_st = nullptr;
        if (hk_use) {
            const unsigned char* hk_got = hk_pipe.acquire(hk_j);
            if (!__all_sync(0xffffffffu, hk_got != nullptr)) break;
            hk_st = hk_got;
        }
        const long long hawk_flat = (hk_t << 8) + static_cast<long long>(threadIdx.x);
        if (hawk_flat < count) {
        const long long hawk_i = base + hawk_flat;
        const hk::SampleIndex i{hawk_i, hk_st, static_cast<int>(threadIdx.x)};
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
        if (hk_use) {
            hk_pipe.release(hk_j);
            if (threadIdx.x == 0 && hk_j + 2 < hk_staged)
                hk_ok = hk_pipe.fill(hk_j + 2, [&](unsigned char* a, unsigned long long* b) { hk_issue(hk_j + 2, a, b); });
            hk_ok = __shfl_sync(0xffffffffu, hk_ok, 0);
        }
    }
    if (threadIdx.x == 0) hk_pipe.drain();
}
