"""Parity at the benchmark configurations' full sizes, through the C ABI.

The ragged-size tests (test_gpu_parity.py) stop at 65553 samples; these run
every configuration's kernels at the size it is benchmarked at and compare
every output with the CPU oracle on all host threads:

  c1 energy fwd / VJP / JVP         2^24 samples
  c2 poly_loss fwd + Param VJP      2^26 samples, float64 and float32
  c3 gravity fwd / JVP / VJP        2^23 samples
  c4 spd_solve fwd / VJP            2^20 samples
  c5 kepler fwd / VJP               2^24 samples (test_gpu_parity.py)

The bar is the north star's -- 1e-12 relative (float64), 1e-5 (float32),
int32 exact -- and every comparison here asserts more: bit-identical outputs
and cells (``same``), as the ragged tests do.
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
THREADS = max(1, min(32, os.cpu_count() or 1))


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def empty(shape, dtype=torch.float64):
    return torch.full(shape, float("nan"), dtype=dtype, device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def same(got, want, what=""):
    got, want = np.asarray(got), np.asarray(want)
    if not np.array_equal(got, want, equal_nan=True):
        rtol = 1e-5 if got.dtype == np.float32 else 1e-12
        np.testing.assert_allclose(got, want, rtol=rtol, err_msg=what)
        differ = int((got != want).sum())
        raise AssertionError(f"{what}: within {rtol} but {differ} values not bit-identical to the oracle")


def test_energy_full_size():
    n = workloads.FULL_N["energy"]
    w = workloads.energy(n, seed=101)
    v = dev(w["v"])
    out = empty((n,))
    runtime.run(runtime.load(BUNDLES, "energy"), v=v, out=out)
    same(host(out), oracle.energy(w["v"], threads=THREADS), "energy")
    del out
    bar_v = empty((3, n))
    runtime.run(runtime.load(BUNDLES, "energy_vjp"), v=v, bar_out=dev(w["bar_out"]), bar_v=bar_v)
    same(host(bar_v), oracle.energy_vjp(w["v"], w["bar_out"], threads=THREADS), "energy_vjp")
    del bar_v
    dot_out = empty((n,))
    runtime.run(runtime.load(BUNDLES, "energy_jvp"), v=v, dot_v=dev(w["dot_v"]), dot_out=dot_out)
    same(host(dot_out), oracle.energy_jvp(w["v"], w["dot_v"], threads=THREADS), "energy_jvp")


@pytest.mark.parametrize("mode,dtype", [("float64", np.float64), ("float32", np.float32)])
def test_poly_loss_full_size(mode, dtype):
    n = workloads.FULL_N["poly_loss"]
    w = workloads.poly_loss(n, seed=102, dtype=dtype)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    x, t = dev(w["x"]), dev(w["t"])
    r = empty((n,), tdt)
    runtime.run(runtime.load(BUNDLES, "poly_loss", mode), x=x, t=t, a=w["a"], b=w["b"], c=w["c"], r=r)
    want = oracle.poly_loss(w["x"], w["t"], dtype(w["a"]), dtype(w["b"]), dtype(w["c"]), threads=THREADS)
    same(host(r), want, f"poly_loss.{mode}")
    del r
    cells = {k: empty((1,), tdt) for k in ("bar_a", "bar_b", "bar_c")}
    abc = {k: dev(np.array([w[k]], dtype=dtype)) for k in ("a", "b", "c")}
    runtime.run(runtime.load(BUNDLES, "poly_loss_vjp", mode), x=x, t=t, bar_r=dev(w["bar_r"]), **abc, **cells)
    want_cells, _rows = oracle.poly_loss_vjp(w["x"], w["t"], w["bar_r"], dtype(w["a"]), dtype(w["b"]),
                                             dtype(w["c"]), threads=THREADS)
    got = [host(cells[k])[0] for k in ("bar_a", "bar_b", "bar_c")]
    assert got == [dtype(v) for v in want_cells], (got, want_cells)


def test_gravity_full_size():
    n = workloads.FULL_N["gravity"]
    w = workloads.gravity(n, seed=103)
    r1, r2, m1, m2 = dev(w["r1"]), dev(w["r2"]), dev(w["m1"]), dev(w["m2"])
    f, u = empty((3, n)), empty((n,))
    runtime.run(runtime.load(BUNDLES, "gravity"), r1=r1, r2=r2, m1=m1, m2=m2, G=w["G"], f=f, u=u)
    wf, wu = oracle.gravity(w["r1"], w["r2"], w["m1"], w["m2"], w["G"], threads=THREADS)
    same(host(f), wf, "gravity f")
    same(host(u), wu, "gravity u")
    df, du = f, u
    runtime.run(runtime.load(BUNDLES, "gravity_jvp"), r1=r1, r2=r2, dot_r1=dev(w["dr1"]), dot_r2=dev(w["dr2"]),
                m1=m1, m2=m2, G=w["G"], dot_f=df, dot_u=du)
    wdf, wdu = oracle.gravity_jvp(w["r1"], w["r2"], w["dr1"], w["dr2"], w["m1"], w["m2"], w["G"], threads=THREADS)
    same(host(df), wdf, "gravity_jvp dot_f")
    same(host(du), wdu, "gravity_jvp dot_u")
    b1, b2 = empty((3, n)), empty((3, n))
    runtime.run(runtime.load(BUNDLES, "gravity_vjp"), r1=r1, r2=r2, bar_f=dev(w["bar_f"]), bar_u=dev(w["bar_u"]),
                m1=m1, m2=m2, G=w["G"], bar_r1=b1, bar_r2=b2)
    wb1, wb2 = oracle.gravity_vjp(w["r1"], w["r2"], w["bar_f"], w["bar_u"], w["m1"], w["m2"], w["G"],
                                  threads=THREADS)
    same(host(b1), wb1, "gravity_vjp bar_r1")
    same(host(b2), wb2, "gravity_vjp bar_r2")


def test_spd_solve_full_size():
    n = workloads.FULL_N["spd_solve"]
    w = workloads.spd_solve(n, seed=104)
    A, b = dev(w["A"]), dev(w["b"])
    x = empty((6, n))
    runtime.run(runtime.load(BUNDLES, "spd_solve"), A=A, b=b, x=x)
    same(host(x), oracle.spd_solve(w["A"], w["b"], threads=THREADS), "spd_solve")
    bar_A, bar_b = empty((6, 6, n)), empty((6, n))
    runtime.run(runtime.load(BUNDLES, "spd_solve_vjp"), A=A, b=b, bar_x=dev(w["bar_x"]), bar_A=bar_A, bar_b=bar_b)
    wA, wb = oracle.spd_solve_vjp(w["A"], w["b"], w["bar_x"], threads=THREADS)
    same(host(bar_A), wA, "spd_solve_vjp bar_A")
    same(host(bar_b), wb, "spd_solve_vjp bar_b")
