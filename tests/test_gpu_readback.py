"""Sums over samples read back in the body, on the B200.

``z = x / hawk.sum(x)`` needs every sample's x before any sample's z, so the
reference's split (hawk/ir/split.py) runs it as stages: the first reduces into
32-sample rows, the rows are finished into the cell, the next stage reads the
cell as a one-cell plane.  The b200 runtime finishes the rows on the device
between the launches with the reference's ordered tree, so every value equals
the CPU oracle's (the host frame's rows, hawk/_cells.py's finish, the bodies'
operations) bit for bit -- the tolerance the north star states (1e-12
relative) is asserted beside the exact comparison.  Sizes are the reference's
ragged cases (tests/test_split_stages.py SIZES) and one past a 4096-row leaf.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from hawk_b200 import runtime  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
SIZES = [1, 31, 33, 1000, 65536, 131072 * 2 + 17]


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def nan(shape):
    return torch.full(shape if isinstance(shape, tuple) else (shape,), float("nan"), dtype=torch.float64, device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def exact(got, want):
    np.testing.assert_array_equal(got, want)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=0)


@pytest.mark.parametrize("n", SIZES)
def test_share_is_two_stages_with_the_cell_finished_between(n):
    x = np.random.default_rng(n).uniform(0.5, 1.5, n)
    z = nan(n)
    runtime.run(runtime.load(BUNDLES, "share"), x=dev(x), z=z)
    exact(host(z), oracle.share(x))


@pytest.mark.parametrize("n", SIZES)
def test_standard_stores_its_mean_and_sum_of_squares(n):
    x = np.random.default_rng(n + 1).normal(3.0, 2.0, n)
    mu, z, t = nan(1), nan(n), nan(1)
    runtime.run(runtime.load(BUNDLES, "standard"), x=dev(x), mu=mu, z=z, t=t)
    want_mu, want_z, want_t = oracle.standard(x)
    exact(host(mu)[0], want_mu)
    if n > 1:
        exact(host(z), want_z)
        exact(host(t)[0], want_t)


@pytest.mark.parametrize("n", SIZES)
def test_a_vector_mean_is_read_back_column_by_column(n):
    x = np.random.default_rng(n + 2).normal(0.0, 1.0, n)
    z = nan((3, n))
    runtime.run(runtime.load(BUNDLES, "centred"), x=dev(x), z=z)
    exact(host(z), oracle.centred(x))


@pytest.mark.parametrize("n", SIZES)
def test_the_vjp_of_a_split_kernel_is_split_too(n):
    rng = np.random.default_rng(n + 3)
    x, bar_z = rng.uniform(0.5, 1.5, n), rng.normal(0.0, 1.0, n)
    bar_x = nan(n)
    runtime.run(runtime.load(BUNDLES, "share_vjp"), x=dev(x), bar_z=dev(bar_z), bar_x=bar_x)
    exact(host(bar_x), oracle.share_vjp(x, bar_z))


def test_runs_in_a_row_reuse_the_kernels_own_cells():
    k = runtime.load(BUNDLES, "share")
    for n, seed in ((5000, 1), (5000, 2), (70000, 3)):
        x = np.random.default_rng(seed).uniform(0.5, 1.5, n)
        z = nan(n)
        runtime.run(k, x=dev(x), z=z)
        exact(host(z), oracle.share(x))
