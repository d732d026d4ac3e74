"""The banded scalar mode on the B200.

A banded value on the b200 target is an IEEE binary64 in its 8-byte cell (this
build's own cell format: the reference's packed BandedReal is defined only by
the absent aether-dsc).  Every op is correctly rounded, so within the 0.5 ULP53
a banded op is certified to; the contract the reference's tests hold the mode
to is checked here the same way:

* a sum over a warp row: each row within 0.6 ULP53 of the exact rational sum
  on ordinary data and within 0.01 ULP53 on a series cancelling by 2^30
  (tests/test_banded_sum.py:20, :79-80 of the reference), its companion row
  zero; bit-identical to the oracle's compensated row rounded once;
* max / min over a row: bitwise NumPy's max / min of the terms
  (tests/test_banded_maxmin.py:4-6);
* a mul/add/div chain with two transcendentals: within the sum of its per-op
  bounds, 3 ULP53, of the float64 build (tests/test_banded_end_to_end.py) --
  measured bit-identical;
* the cells finished on the device over the banded rows: bit-identical to the
  oracle's finish of the same rows, and within the rows' rounding of the exact
  total; the Param gradients of the headline VJP built banded likewise.
"""

from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest

import oracle
from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from hawk_b200 import runtime, workloads  # noqa: E402
from hawk_b200.planes import as_plane  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float64), device="cuda")


def ulp53(x: float) -> Fraction:
    return Fraction(float(np.spacing(abs(float(x)))))


def ordinary(n):
    return np.random.default_rng(5).uniform(-2.0, 2.0, n).astype(np.float32).astype(np.float64)


def cancelling(n):
    """Rows of 2^30, 1, -2^30, 1, ...: every term float32-exact, each row's
    exact sum small against its terms."""
    return np.tile([2.0 ** 30, 1.0, -(2.0 ** 30), 1.0], n // 4 + 1)[:n].astype(np.float64)


def exact_rows(x):
    return [sum(Fraction(float(v)) for v in x[r * 32:(r + 1) * 32]) for r in range(-(-x.shape[0] // 32))]


def row_planes(kernel, x, names):
    """Launch ``kernel`` over ``x`` with its row planes bound directly."""
    n = x.shape[0]
    nrows = -(-n // 32)
    out = {name: torch.full((nrows,), float("nan"), dtype=torch.float64, device="cuda") for name in names}
    planes = {"x": dev(x), **out}
    bound = {name: as_plane(name, obj) for name, obj in planes.items()}
    kernel.check(bound, {}, n)
    kernel.bind_all(bound, {}, n)
    kernel.launch(0, n, n)
    torch.cuda.synchronize()
    return {name: t.cpu().numpy() for name, t in out.items()}


@pytest.mark.parametrize("n", [1000, 65536 + 17])
@pytest.mark.parametrize("data,bound", [(ordinary, Fraction(6, 10)), (cancelling, Fraction(1, 100))],
                         ids=["ordinary", "cancelling"])
def test_banded_row_sums_are_within_their_bound_of_the_exact_sum(data, bound, n):
    k = runtime.load(BUNDLES, "band_rows", "banded")
    assert k.mode == "banded" and k.element == "float64"
    x = data(n)
    got = row_planes(k, x, ("s", "s_comp", "q", "q_comp"))
    for name, terms in (("s", x), ("q", x * x)):
        for r, (g, want) in enumerate(zip(got[name], exact_rows(terms))):
            err = abs(Fraction(float(g)) - want) / ulp53(float(want)) if want else abs(Fraction(float(g)))
            assert err <= bound, (name, r, float(g), float(want), float(err))
        np.testing.assert_array_equal(got[name + "_comp"], 0.0)
        want_rows, _zero = oracle.banded_rows(terms)
        np.testing.assert_array_equal(got[name], want_rows)


@pytest.mark.parametrize("name,plane,ref", [("band_max", "hi", np.max), ("band_min", "lo", np.min)])
def test_banded_row_extremes_are_bitwise_numpys(name, plane, ref):
    rng = np.random.default_rng(11)
    n = 1000
    x = rng.uniform(-2.0, 2.0, n) * np.exp2(rng.integers(-20, 20, n))
    x[::97] = 0.0
    x[5::97] = -0.0
    x = x.astype(np.float32).astype(np.float64)
    got = row_planes(runtime.load(BUNDLES, name, "banded"), x, (plane,))[plane]
    want = np.array([ref(x[r * 32:(r + 1) * 32]) for r in range(-(-n // 32))])
    np.testing.assert_array_equal(got.view(np.uint64), want.view(np.uint64))


def test_a_banded_chain_equals_the_float64_build():
    n = 4096
    rng = np.random.default_rng(13)
    x = rng.uniform(-2.0, 2.0, n).astype(np.float32).astype(np.float64)
    y = rng.uniform(0.0, 3.0, n).astype(np.float32).astype(np.float64)
    outs = {}
    for mode in ("banded", "float64"):
        out = torch.full((n,), float("nan"), dtype=torch.float64, device="cuda")
        runtime.run(runtime.load(BUNDLES, "band_chain", mode), x=dev(x), y=dev(y), out=out)
        outs[mode] = out.cpu().numpy()
    diff = np.abs(outs["banded"] - outs["float64"]) / np.spacing(np.abs(outs["float64"]))
    assert diff.max() <= 3.0
    np.testing.assert_array_equal(outs["banded"], outs["float64"])


@pytest.mark.parametrize("n", [1000, 300000])
def test_banded_cells_are_the_finish_of_the_banded_rows(n):
    x = ordinary(n)
    cells = {c: torch.full((1,), float("nan"), dtype=torch.float64, device="cuda") for c in ("s", "q")}
    runtime.run(runtime.load(BUNDLES, "band_rows", "banded"), x=dev(x), **cells)
    for c, terms in (("s", x), ("q", x * x)):
        got = float(cells[c].cpu()[0])
        hi, zero = oracle.banded_rows(terms)
        assert got == oracle.cells_finish(hi, zero)
        exact = sum(Fraction(float(v)) for v in terms)
        slack = sum(ulp53(r) / 2 for r in hi) + ulp53(float(exact)) / 2
        assert abs(Fraction(got) - exact) <= slack * Fraction(11, 10), (c, got, float(exact))


def test_param_gradients_built_banded():
    n = 65536 + 17
    w = workloads.poly_loss(n, seed=8)
    cells = {k: torch.full((1,), float("nan"), dtype=torch.float64, device="cuda") for k in ("bar_a", "bar_b", "bar_c")}
    abc = {k: dev(np.array([w[k]])) for k in ("a", "b", "c")}
    runtime.run(runtime.load(BUNDLES, "poly_loss_vjp", "banded"), x=dev(w["x"]), t=dev(w["t"]),
                bar_r=dev(w["bar_r"]), **abc, **cells)
    hi, comp = oracle.poly_loss_vjp_rows(w["x"], w["t"], w["bar_r"], w["a"], w["b"], w["c"])
    for j, k in enumerate(("bar_a", "bar_b", "bar_c")):
        assert float(cells[k].cpu()[0]) == oracle.cells_finish(hi[j] + comp[j], np.zeros_like(hi[j]))
