"""Sums over some lane axes on the B200: ``hawk.sum(x, over="row")`` over a
``Grid["key", "row":8]`` lane space.

A kernel returning the sum commits each key's total into its output plane (an
aligned run of eight lanes: one butterfly, one commit); a kernel reading it
back runs as the reference's two stages with a keyed plane the runtime owns
between them, zeroed every run (hawk/runtime.py:655-673).  On fully converged
warps (a multiple of 32 lanes) every key's sum is one commit, so the device
equals the oracle bit for bit; a partial last warp commits lane by lane in the
hardware's order, inside the reference's keyed-commit bound
(tests/test_keyed_commit.py).
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from hawk_b200 import runtime  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
EPS = np.finfo(np.float64).eps


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("n", [32, 4096, 262144 + 32])
def test_key_totals_are_one_butterfly_per_key(n):
    x = np.random.default_rng(n).normal(0.0, 1.0, n)
    out = torch.zeros(n // 8, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "key_total"), x=dev(x), out=out)
    np.testing.assert_array_equal(host(out), oracle.key_sums(x))


@pytest.mark.parametrize("n", [8, 40, 1000])
def test_key_totals_of_a_partial_warp_are_within_the_commit_bound(n):
    x = np.random.default_rng(n).normal(0.0, 1.0, n)
    out = torch.zeros(n // 8, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "key_total"), x=dev(x), out=out)
    got = host(out)
    for k in range(n // 8):
        seg = x[8 * k:8 * k + 8]
        assert abs(got[k] - math.fsum(seg)) <= 16 * EPS * math.fsum(np.abs(seg))


@pytest.mark.parametrize("n", [32, 4096, 262144 + 32])
def test_a_keyed_sum_read_back_is_two_stages_over_a_zeroed_keyed_plane(n):
    k = runtime.load(BUNDLES, "key_share")
    for seed in (1, 2):                 # a second run sees the keyed plane zeroed again
        x = np.random.default_rng(n + seed).uniform(0.5, 1.5, n)
        z = torch.full((n,), float("nan"), dtype=torch.float64, device="cuda")
        runtime.run(k, x=dev(x), z=z)
        want = oracle.key_share(x)
        np.testing.assert_array_equal(host(z), want)
        np.testing.assert_allclose(host(z), want, rtol=1e-12)


@pytest.mark.parametrize("keys", [1, 37, 4096])
def test_gram_blocks_are_ordered_sums_per_key(keys):
    """hawk.sum(outer(j, j), over="row") of a 6-vector: a BlockSum (36 entries)
    -- the rows stored by the first stage, each key's 6 x 6 block summed in
    lane order by a team stage -- bit-identical to the oracle's ordered sum."""
    n = 8 * keys
    j = np.random.default_rng(keys).normal(0.0, 1.0, (6, n))
    out = torch.full((6, 6, keys), float("nan"), dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "gram_block"), j=dev(j), out=out)
    np.testing.assert_array_equal(host(out), oracle.block_sums(j, j))


@pytest.mark.parametrize("keys", [3, 1000])
def test_gradient_blocks_are_ordered_sums_per_key(keys):
    n = 8 * keys
    rng = np.random.default_rng(keys + 1)
    j, r = rng.normal(0.0, 1.0, (20, n)), rng.normal(0.0, 1.0, n)
    out = torch.full((20, keys), float("nan"), dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "grad_block"), j=dev(j), r=dev(r), out=out)
    np.testing.assert_array_equal(host(out), oracle.block_sums(j, r[None, :])[:, 0, :])
