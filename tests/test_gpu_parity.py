"""Parity of the b200 device path with the CPU oracle, through the C ABI.

Every kernel runs through ``hawk_b200.runtime`` (load -> bind -> launch on the
B200) on seeded inputs and is compared with the oracle on the same inputs.
The tolerance is the north star's -- 1e-12 relative (float64), 1e-5 (float32),
exact for int32 planes -- and the device is asserted bit-identical to the
oracle where the design makes it so: both evaluate the same operations in the
same order without FMA contraction, with correctly rounded division and sqrt.

Sizes mirror the reference's ragged cases (tests/test_sample_sum.py:36):
1, 31, 32, 33, 1000 and 65536 + 17; outputs are NaN-prefilled so an unwritten
sample shows.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from hawk_b200 import runtime, workloads  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
SIZES = [1, 31, 32, 33, 1000, 65536 + 17]


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def nan_like(shape, dtype=torch.float64):
    return torch.full(shape, float("nan"), dtype=dtype, device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def same(got, want):
    """Bit-identical (NaN-aware), with the 1e-12 tolerance reported on failure."""
    got, want = np.asarray(got), np.asarray(want)
    if not np.array_equal(got, want, equal_nan=True):
        np.testing.assert_allclose(got, want, rtol=1e-12)
        raise AssertionError("within 1e-12 but not bit-identical to the oracle")


@pytest.mark.parametrize("n", SIZES)
def test_energy_fwd_vjp_jvp(n):
    w = workloads.energy(n, seed=n)
    v = dev(w["v"])
    out = nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "energy"), v=v, out=out)
    same(host(out), oracle.energy(w["v"]))
    bar_v = nan_like((3, n))
    runtime.run(runtime.load(BUNDLES, "energy_vjp"), v=v, bar_out=dev(w["bar_out"]), bar_v=bar_v)
    same(host(bar_v), oracle.energy_vjp(w["v"], w["bar_out"]))
    dot_out = nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "energy_jvp"), v=v, dot_v=dev(w["dot_v"]), dot_out=dot_out)
    same(host(dot_out), oracle.energy_jvp(w["v"], w["dot_v"]))


def test_energy_known_answer():
    v = dev([[1.0, 2.0, 3.0, 4.0], [0.0, 1.0, 0.0, 1.0], [0.0, 0.0, 1.0, 1.0]])
    out = nan_like((4,))
    runtime.run(runtime.load(BUNDLES, "energy"), v=v, out=out)
    np.testing.assert_array_equal(host(out), [0.5, 2.5, 5.0, 9.0])
    bar_v = nan_like((3, 4))
    runtime.run(runtime.load(BUNDLES, "energy_vjp"), v=v, bar_out=dev(np.ones(4)), bar_v=bar_v)
    np.testing.assert_array_equal(host(bar_v), host(v))


@pytest.mark.parametrize("mode,dtype", [("float64", np.float64), ("float32", np.float32)])
@pytest.mark.parametrize("n", SIZES)
def test_poly_loss_fwd_and_param_gradients(n, mode, dtype):
    w = workloads.poly_loss(n, seed=n, dtype=dtype)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    x, t, bar_r = dev(w["x"]), dev(w["t"]), dev(w["bar_r"])
    r = nan_like((n,), tdt)
    fwd = runtime.load(BUNDLES, "poly_loss", mode)
    runtime.run(fwd, x=x, t=t, a=w["a"], b=w["b"], c=w["c"], r=r)
    want = oracle.poly_loss(w["x"], w["t"], dtype(w["a"]), dtype(w["b"]), dtype(w["c"]))
    same(host(r), want)
    cells = {k: nan_like((1,), tdt) for k in ("bar_a", "bar_b", "bar_c")}
    vjp = runtime.load(BUNDLES, "poly_loss_vjp", mode)
    abc = {k: dev(np.array([w[k]], dtype=dtype)) for k in ("a", "b", "c")}
    runtime.run(vjp, x=x, t=t, bar_r=bar_r, **abc, **cells)
    want_cells, _rows = oracle.poly_loss_vjp(w["x"], w["t"], w["bar_r"], dtype(w["a"]), dtype(w["b"]),
                                             dtype(w["c"]))
    got = [host(cells[k])[0] for k in ("bar_a", "bar_b", "bar_c")]
    # the rows and the finish tree are the oracle's operations in the oracle's order
    assert got == [dtype(v) for v in want_cells], (got, want_cells)


def test_poly_loss_rows_through_the_entry():
    """The VJP entry bound directly to row planes (the reference's param_planes
    test form, tests/test_param_planes.py:150-178): rows equal the oracle's."""
    n = 5000
    w = workloads.poly_loss(n, seed=3)
    k = runtime.load(BUNDLES, "poly_loss_vjp")
    rows = -(-n // 32)
    planes = {name: dev(w[name]) for name in ("x", "t", "bar_r")}
    planes.update({name: dev(np.array([w[name]])) for name in ("a", "b", "c")})
    out = {name: nan_like((rows,)) for name in ("bar_a", "bar_a_comp", "bar_b", "bar_b_comp", "bar_c", "bar_c_comp")}
    from hawk_b200.planes import as_plane
    bound = {name: as_plane(name, obj) for name, obj in {**planes, **out}.items()}
    k.check(bound, {}, n)
    k.bind_all(bound, {}, n)
    k.launch(0, n, n)
    hi, comp = oracle.poly_loss_vjp_rows(w["x"], w["t"], w["bar_r"], w["a"], w["b"], w["c"])
    for j, name in enumerate(("bar_a", "bar_b", "bar_c")):
        same(host(out[name]), hi[j])
        same(host(out[name + "_comp"]), comp[j])


@pytest.mark.parametrize("shift,n,base", [(0, 256 * 37, 0), (0, 256 * 37 + 1, 0), (0, 256 * 37 - 1, 0),
                                          (1, 5000, 0), (0, 40000, 4096), (1, 40000, 4096)],
                         ids=["whole-tiles", "one-past", "one-short", "unaligned", "partition", "unaligned-partition"])
def test_warp_tiled_rows_match_the_oracle(shift, n, base):
    """The VJP's row frame fetches each warp's next trip into its shared-memory
    tile (``warp_tiled`` in the sidecar): whole trips come from the tile, a
    partial last trip and planes off the 16-byte boundary (``shift`` of one
    element: every trip) from global memory.  Every row of the partition
    equals the oracle's, rows outside it are untouched, and no bounded wait
    ran out."""
    import warnings

    from hawk_b200.planes import as_plane

    k = runtime.load(BUNDLES, "poly_loss_vjp")
    assert k.sidecar["b200"]["warp_tiled"]
    w = workloads.poly_loss(n, seed=n + shift)

    def shifted(a):
        t = torch.empty(len(a) + shift, dtype=torch.float64, device="cuda")
        t[shift:] = dev(a)
        return t[shift:]

    rows = -(-n // 32)
    planes = {name: shifted(w[name]) for name in ("x", "t", "bar_r")}
    planes.update({name: dev(np.array([w[name]])) for name in ("a", "b", "c")})
    out = {name: nan_like((rows,)) for name in ("bar_a", "bar_a_comp", "bar_b", "bar_b_comp", "bar_c", "bar_c_comp")}
    bound = {name: as_plane(name, obj) for name, obj in {**planes, **out}.items()}
    k.check(bound, {}, n)
    k.bind_all(bound, {}, n)
    k.launch(base, n - base, n)
    torch.cuda.synchronize()
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        k.check_waits()
    hi, comp = oracle.poly_loss_vjp_rows(w["x"], w["t"], w["bar_r"], w["a"], w["b"], w["c"])
    lo = base // 32
    for j, name in enumerate(("bar_a", "bar_b", "bar_c")):
        got_hi, got_comp = host(out[name]), host(out[name + "_comp"])
        assert np.isnan(got_hi[:lo]).all() and np.isnan(got_comp[:lo]).all()
        same(got_hi[lo:], hi[j, lo:])
        same(got_comp[lo:], comp[j, lo:])


@pytest.mark.parametrize("n", SIZES)
def test_gravity_fwd_jvp_vjp(n):
    w = workloads.gravity(n, seed=n)
    r1, r2, m1, m2 = dev(w["r1"]), dev(w["r2"]), dev(w["m1"]), dev(w["m2"])
    f, u = nan_like((3, n)), nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "gravity"), r1=r1, r2=r2, m1=m1, m2=m2, G=w["G"], f=f, u=u)
    wf, wu = oracle.gravity(w["r1"], w["r2"], w["m1"], w["m2"], w["G"])
    same(host(f), wf)
    same(host(u), wu)
    df, du = nan_like((3, n)), nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "gravity_jvp"), r1=r1, r2=r2, dot_r1=dev(w["dr1"]), dot_r2=dev(w["dr2"]),
                m1=m1, m2=m2, G=w["G"], dot_f=df, dot_u=du)
    wdf, wdu = oracle.gravity_jvp(w["r1"], w["r2"], w["dr1"], w["dr2"], w["m1"], w["m2"], w["G"])
    same(host(df), wdf)
    same(host(du), wdu)
    b1, b2 = nan_like((3, n)), nan_like((3, n))
    runtime.run(runtime.load(BUNDLES, "gravity_vjp"), r1=r1, r2=r2, bar_f=dev(w["bar_f"]), bar_u=dev(w["bar_u"]),
                m1=m1, m2=m2, G=w["G"], bar_r1=b1, bar_r2=b2)
    wb1, wb2 = oracle.gravity_vjp(w["r1"], w["r2"], w["bar_f"], w["bar_u"], w["m1"], w["m2"], w["G"])
    same(host(b1), wb1)
    same(host(b2), wb2)


@pytest.mark.parametrize("n", SIZES)
def test_spd_solve_fwd_vjp(n):
    w = workloads.spd_solve(n, seed=n)
    A, b = dev(w["A"]), dev(w["b"])
    x = nan_like((6, n))
    runtime.run(runtime.load(BUNDLES, "spd_solve"), A=A, b=b, x=x)
    same(host(x), oracle.spd_solve(w["A"], w["b"]))
    bar_A, bar_b = nan_like((6, 6, n)), nan_like((6, n))
    runtime.run(runtime.load(BUNDLES, "spd_solve_vjp"), A=A, b=b, bar_x=dev(w["bar_x"]), bar_A=bar_A, bar_b=bar_b)
    wA, wb = oracle.spd_solve_vjp(w["A"], w["b"], w["bar_x"])
    same(host(bar_A), wA)
    same(host(bar_b), wb)


def test_spd_solve_failed_factor_solves_to_zeros():
    n = 64
    w = workloads.spd_solve(n, seed=1)
    A = w["A"].copy()
    A[2, 2, 5] = -1.0e6          # sample 5: not positive definite -> info > 0 -> zeros
    x = nan_like((6, n))
    runtime.run(runtime.load(BUNDLES, "spd_solve"), A=dev(A), b=dev(w["b"]), x=x)
    got = host(x)
    same(got, oracle.spd_solve(A, w["b"]))
    np.testing.assert_array_equal(got[:, 5], np.zeros(6))


@pytest.mark.parametrize("n", SIZES)
def test_kepler_fwd_vjp(n):
    w = workloads.kepler(n, seed=n)
    e, M = dev(w["e"]), dev(w["M"])
    E, it = nan_like((n,)), torch.full((n,), -1, dtype=torch.int32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "kepler"), e=e, M=M, E=E, iters=it)
    wE, wit = oracle.kepler(w["e"], w["M"])
    wbe, wbM = oracle.kepler_vjp(w["e"], w["M"], w["bar_E"])
    np.testing.assert_array_equal(host(it), wit)           # int32 plane: bit-exact
    same(host(E), wE)
    be, bM = nan_like((n,)), nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "kepler_vjp"), e=e, M=M, bar_E=dev(w["bar_E"]), bar_e=be, bar_M=bM)
    same(host(be), wbe)
    same(host(bM), wbM)


def trig_arguments(seed: int) -> np.ndarray:
    """Arguments over every range of glibc's sin/cos method, with its range
    boundaries and special values."""
    rng = np.random.default_rng(seed)
    x = np.concatenate([rng.uniform(-0.126, 0.126, 1 << 20), rng.uniform(-8.0, 8.0, 1 << 22),
                        rng.uniform(-105414350.0, 105414350.0, 1 << 20),
                        np.ldexp(rng.uniform(1, 2, 1 << 18), rng.integers(27, 1024, 1 << 18)),
                        np.ldexp(rng.uniform(1, 2, 1 << 16), rng.integers(-1074, -20, 1 << 16)),
                        [0.0, -0.0, 2.0 ** -1074, 2.0 ** -27, 2.0 ** -26, 0.126, 0.85546875, 2.426265,
                         105414350.0, 1e22, 6381956970095103.0 * 2.0 ** 797, 1.7976931348623157e308,
                         np.inf, -np.inf, np.nan]])
    sign = rng.integers(0, 2, x.shape[0]) * 2 - 1
    return x * sign


def test_trig_has_glibcs_bits():
    """sin and cos on the device against the host's glibc (the reference host
    target's libm) on 6.4 million arguments over every range of its method,
    the large-argument reduction and the special values: bit-identical."""
    x = trig_arguments(17)
    n = x.shape[0]
    s, c = nan_like((n,)), nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "trig"), x=dev(x), s=s, c=c)
    ws, wc = oracle.trig(x, threads=max(1, min(32, os.cpu_count() or 1)))
    same(host(s), ws)
    same(host(c), wc)


@pytest.mark.parametrize("seed", [11, 12])
def test_kepler_full_size_against_the_glibc_oracle(seed):
    """The configuration's full size, 2^24 samples: the int32 iteration counts
    equal the reference host target's (glibc's sin/cos) on every sample, and E
    and the VJP bit-identical to it."""
    n = workloads.FULL_N["kepler"]
    w = workloads.kepler(n, seed=seed)
    e, M = dev(w["e"]), dev(w["M"])
    E, it = nan_like((n,)), torch.full((n,), -1, dtype=torch.int32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "kepler"), e=e, M=M, E=E, iters=it)
    threads = max(1, min(32, os.cpu_count() or 1))
    wE, wit = oracle.kepler(w["e"], w["M"], threads=threads)
    assert int((host(it) != wit).sum()) == 0
    same(host(E), wE)
    be, bM = nan_like((n,)), nan_like((n,))
    runtime.run(runtime.load(BUNDLES, "kepler_vjp"), e=e, M=M, bar_E=dev(w["bar_E"]), bar_e=be, bar_M=bM)
    wbe, wbM = oracle.kepler_vjp(w["e"], w["M"], w["bar_E"], threads=threads)
    same(host(be), wbe)
    same(host(bM), wbM)


def test_kepler_beyond_two_to_the_twenty():
    """Mean anomalies from 2^20 to 1e300 (sin/cos through both argument
    reductions), infinities and NaN: bit-identical to the glibc oracle,
    iteration counts included."""
    rng = np.random.default_rng(5)
    # below 2^52 or so e*sin(E) still moves E, so the exact sin/cos bits show
    M = np.concatenate([np.ldexp(rng.uniform(1, 2, 4000), rng.integers(20, 52, 4000)),
                        np.ldexp(rng.uniform(1, 2, 1000), rng.integers(52, 997, 1000)),
                        [1048576.0, 1048577.5, 6381956970095103.0 * 2.0 ** 797, 1e300, np.inf, -np.inf, np.nan]])
    e = rng.uniform(0, 0.95, M.shape[0])
    n = M.shape[0]
    E, it = nan_like((n,)), torch.full((n,), -1, dtype=torch.int32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "kepler"), e=dev(e), M=dev(M), E=E, iters=it)
    wE, wit = oracle.kepler(e, M)
    np.testing.assert_array_equal(host(it), wit)
    same(host(E), wE)


def test_kepler_known_answer():
    E, it = nan_like((1,)), torch.full((1,), -1, dtype=torch.int32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "kepler"), e=dev([0.5]), M=dev([1.0]), E=E, iters=it)
    assert host(E)[0] == 1.4987011335178484 and host(it)[0] == 6


def test_partition_writes_only_its_samples():
    """``base``/``count`` (the partition triple): samples outside stay untouched."""
    n = 10000
    w = workloads.energy(n, seed=5)
    out = nan_like((n,))
    k = runtime.load(BUNDLES, "energy")
    runtime.run(k, v=dev(w["v"]), out=out, base=1234, count=5000)
    got = host(out)
    want = oracle.energy(w["v"])
    assert np.isnan(got[:1234]).all() and np.isnan(got[6234:]).all()
    same(got[1234:6234], want[1234:6234])


def test_cells_over_a_partition_and_a_refused_unaligned_base():
    n = 40000
    w = workloads.poly_loss(n, seed=9)
    k = runtime.load(BUNDLES, "poly_loss_vjp")
    planes = {name: dev(w[name]) for name in ("x", "t", "bar_r")}
    planes.update({name: dev(np.array([w[name]])) for name in ("a", "b", "c")})
    cells = {c: nan_like((1,)) for c in ("bar_a", "bar_b", "bar_c")}
    runtime.run(k, base=4096, count=20000, **planes, **cells)
    hi, comp = oracle.poly_loss_vjp_rows(w["x"], w["t"], w["bar_r"], w["a"], w["b"], w["c"])
    lo, hi_row = 4096 // 32, -(-(4096 + 20000) // 32)
    for j, c in enumerate(("bar_a", "bar_b", "bar_c")):
        assert host(cells[c])[0] == oracle.cells_finish(hi[j, lo:hi_row], comp[j, lo:hi_row])
    from hawk_b200.errors import HawkError
    with pytest.raises(HawkError, match="base % 32"):
        runtime.run(k, base=100, count=1000, **planes, **cells)


def test_bind_refusals_name_every_argument():
    from hawk_b200.errors import HawkError
    k = runtime.load(BUNDLES, "gravity")
    n = 100
    w = workloads.gravity(n, seed=1)
    good = dict(r1=dev(w["r1"]), r2=dev(w["r2"]), m1=dev(w["m1"]), m2=dev(w["m2"]), G=1.0,
                f=nan_like((3, n)), u=nan_like((n,)))
    with pytest.raises(HawkError, match="2 arguments failed"):
        runtime.run(k, **{**good, "m1": dev(w["m1"].astype(np.float32)), "f": nan_like((4, n))})
    with pytest.raises(HawkError, match="host array"):
        runtime.run(k, **{**good, "r1": w["r1"]})
    with pytest.raises(HawkError, match="not planes it declares"):
        runtime.run(k, **good, bogus=nan_like((n,)))
    with pytest.raises(HawkError, match="disagree"):
        runtime.run(k, **{**good, "u": nan_like((n + 1,))})


STAGED = BUNDLES / "staged"


@pytest.mark.parametrize("n", [1, 33, 1000, 65536 + 17, 300000])
def test_staged_units_match_the_oracle(n):
    """The shared-memory staged entries (cp.async.bulk into stages, mbarrier
    waits): the SPD VJP (lane frame) and the Param-gradient VJP (row frame)
    bit-identical to the oracle, with the unit's error word still clear."""
    w = workloads.spd_solve(n, seed=n + 1)
    k = runtime.load(STAGED, "spd_solve_vjp")
    assert k.sidecar["b200"]["stages"] >= 2
    bar_A, bar_b = nan_like((6, 6, n)), nan_like((6, n))
    runtime.run(k, A=dev(w["A"]), b=dev(w["b"]), bar_x=dev(w["bar_x"]), bar_A=bar_A, bar_b=bar_b)
    wA, wb = oracle.spd_solve_vjp(w["A"], w["b"], w["bar_x"])
    same(host(bar_A), wA)
    same(host(bar_b), wb)
    assert k.library.errors() == 0
    p = workloads.poly_loss(n, seed=n + 2)
    v = runtime.load(STAGED, "poly_loss_vjp")
    cells = {c: nan_like((1,)) for c in ("bar_a", "bar_b", "bar_c")}
    abc = {c: dev(np.array([p[c]])) for c in ("a", "b", "c")}
    runtime.run(v, x=dev(p["x"]), t=dev(p["t"]), bar_r=dev(p["bar_r"]), **abc, **cells)
    want, _rows = oracle.poly_loss_vjp(p["x"], p["t"], p["bar_r"], p["a"], p["b"], p["c"])
    assert [host(cells[c])[0] for c in ("bar_a", "bar_b", "bar_c")] == [float(x) for x in want]
    assert v.library.errors() == 0
