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

Under ``policy="ordered"`` a per-key sum and a scatter by any key run as the
reference's ordered stages (hawk/ir/team.py:602-736): a fixed grouping that
depends on the lane count only, the same bits on every launch, bit-identical
to the oracle (itself pinned bitwise to the reference's numpy emulation of the
grouping by tests/test_oracle_golden.py).
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
from hawk_b200.errors import HawkError  # noqa: E402

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


def ordered_draw(rows: int, keys: int) -> np.ndarray:
    n = rows * keys
    return np.random.default_rng(n).normal(size=n) * np.exp(np.random.default_rng(n + 1).normal(size=n))


@pytest.mark.parametrize("name,rows,keys", [("ordered_total", 8, 5), ("ordered_total", 8, 4096),
                                            ("ordered_long", 197385, 2)])
def test_ordered_sums_are_the_fixed_tree_and_replay_bitwise(name, rows, keys):
    """65536 virtual lanes a key, groups of 1024 by the halving tree, the 64
    group values by the same tree: three launches, one set of bits, the
    oracle's (197385 rows: three strides of 65536 and a partial fourth)."""
    x = ordered_draw(rows, keys)
    k = runtime.load(BUNDLES, name)
    runs = []
    for _ in range(3):
        out = torch.full((keys,), float("nan"), dtype=torch.float64, device="cuda")
        runtime.run(k, x=dev(x), out=out)
        runs.append(host(out))
    assert runs[0].tobytes() == runs[1].tobytes() == runs[2].tobytes()
    np.testing.assert_array_equal(runs[0], oracle.ordered_sums(x, rows))
    assert k.errors() == 0


def scatter_case(n, cells, seed, heavy=False):
    rng = np.random.default_rng(seed)
    key = rng.integers(0, cells, n).astype(np.int32)
    if heavy:
        key[rng.random(n) < 0.9] = cells // 2
    key[::7] = -1
    x = rng.normal(size=n) * np.exp(rng.normal(size=n))
    return key, x


def scatter(key, x, acc, **kw):
    acc = dev(acc)
    runtime.run(runtime.load(BUNDLES, "ordered_hist"), key=dev(key), x=dev(x), acc=acc, **kw)
    return host(acc)


@pytest.mark.parametrize("n,cells,heavy", [(20000, 7, True), (3000, 1, False), (5000, 40, False),
                                           (50, 200, False), (1000, 1000, False), (30000, 1500, False),
                                           (1 << 20, 1000, False)])
def test_ordered_scatter_is_the_chunk_walk_bitwise_and_replays(n, cells, heavy):
    """Heavy collisions (256 chunks on a few cells), one cell, more cells than
    lanes (one chunk), a cell per lane, more cells than the shared bins hold
    (1500: the serial walk) and 2^20 lanes: the oracle's bits, three launches
    alike, and onto a plane that held values the same sums added on top."""
    key, x = scatter_case(n, cells, seed=n + cells, heavy=heavy)
    want, bad = oracle.ordered_scatter(key, x, np.zeros(cells))
    assert not bad
    runs = [scatter(key, x, np.zeros(cells)) for _ in range(3)]
    assert runs[0].tobytes() == runs[1].tobytes() == runs[2].tobytes()
    np.testing.assert_array_equal(runs[0], want)
    base = np.linspace(1.0, 2.0, cells)
    np.testing.assert_array_equal(scatter(key, x, base), oracle.ordered_scatter(key, x, base)[0])


def test_poisoned_partial_sums_do_not_change_the_ordered_scatter():
    """The partial-sum plane is zeroed by the first team stage every launch:
    NaN left in it by anything before does not reach the cells."""
    n, cells = 20000, 7
    key, x = scatter_case(n, cells, seed=3)
    k = runtime.load(BUNDLES, "ordered_hist")
    planes = k.scratch(n, {"acc": cells})
    planes["tms_acc_p"].fill_(float("nan"))
    planes["tms_acc_v"].fill_(float("nan"))
    np.testing.assert_array_equal(scatter(key, x, np.zeros(cells)), oracle.ordered_scatter(key, x, np.zeros(cells))[0])


def test_a_partition_of_the_lanes_adds_only_its_lanes():
    n, cells = 6000, 33
    key, x = scatter_case(n, cells, seed=5)
    got = scatter(key, x, np.zeros(cells), base=1000, count=3000)
    only = np.full(n, -1, np.int32)
    only[1000:4000] = key[1000:4000]
    np.testing.assert_array_equal(got, oracle.ordered_scatter(only, x, np.zeros(cells))[0])
    # the next full launch sees none of the partition's keys left behind
    np.testing.assert_array_equal(scatter(key, x, np.zeros(cells)), oracle.ordered_scatter(key, x, np.zeros(cells))[0])


def test_a_key_out_of_range_is_reported_by_name_and_the_next_launch_is_clean():
    n, cells = 4000, 9
    key, x = scatter_case(n, cells, seed=29)
    for bad in (cells, cells + 5, -2, 2**31 - 2):
        wild = key.copy()
        wild[[3, n - 1]] = bad
        with pytest.raises(HawkError, match=r"hawk.scatter\(acc, policy='ordered'\) got a key outside \[0, 9\)"):
            scatter(wild, x, np.zeros(cells))
    np.testing.assert_array_equal(scatter(key, x, np.zeros(cells)), oracle.ordered_scatter(key, x, np.zeros(cells))[0])


def test_a_target_of_no_cells_reports_any_key_but_the_skip_key():
    n = 300
    x = np.ones(n)
    scatter(np.full(n, -1, np.int32), x, np.zeros(0))
    key = np.full(n, -1, np.int32)
    key[17] = 0
    with pytest.raises(HawkError, match=r"got a key outside \[0, 0\)"):
        scatter(key, x, np.zeros(0))
    scatter(np.full(n, -1, np.int32), x, np.zeros(0))


def test_an_ordered_scatter_of_no_lanes_leaves_the_target_as_it_was():
    acc = np.linspace(1.0, 2.0, 9)
    got = scatter(np.zeros(0, np.int32), np.zeros(0), acc)
    np.testing.assert_array_equal(got, acc)
    np.testing.assert_array_equal(got, oracle.ordered_scatter(np.zeros(0, np.int32), np.zeros(0), acc)[0])


def test_an_ordered_sum_over_no_keys_runs_no_team():
    out = torch.zeros(0, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "ordered_total"), x=dev(np.zeros(0)), out=out)
    assert host(out).shape == (0,)
