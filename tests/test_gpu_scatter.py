"""Scattered commits and table reads on the B200.

Many samples add into one slot, through the device's atomics, so the order of
the adds is the hardware's; the contract is the reference's
(tests/test_keyed_commit.py of the reference): per slot, the error against the
exact sum (``math.fsum`` of the same rounded terms) is within a bound of
eps * sum|t| -- about one for a compensated commit (the default policy's
runtime-owned companion included, folded into the target after the launch),
growing with the terms per slot for a plain one.  Table reads (clamped
indices), their plain adjoint scatter and the OR commit are checked exactly.
Sizes are the reference's ragged cases; partitions and prior slot values are
covered.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from hawk_b200 import runtime, workloads  # noqa: E402
from hawk_b200.workloads import SEGMENT  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
SIZES = [1, 33, 1000, 65536 + 17]
EPS = np.finfo(np.float64).eps


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def exact(keys, terms, slots, prior=None):
    """Per slot: the exact sum (fsum) of the prior value and its terms, sum|t|,
    and the number of terms."""
    groups = [[] for _ in range(slots)]
    for k, t in zip(keys.tolist(), terms.tolist()):
        groups[k].append(t)
    base = np.zeros(slots) if prior is None else prior
    want = np.array([math.fsum([base[s], *g]) for s, g in enumerate(groups)])
    mag = np.array([math.fsum([abs(base[s]), *map(abs, g)]) for s, g in enumerate(groups)])
    cnt = np.array([len(g) for g in groups])
    return want, mag, cnt


def within(got, want, mag, factor):
    err = np.abs(got - want)
    ok = err <= factor * EPS * mag
    assert ok.all(), (np.flatnonzero(~ok)[:5], (err / np.maximum(mag, 1e-300))[~ok][:5] / EPS)


@pytest.mark.parametrize("n", SIZES)
def test_gather_reads_clamped_table_slots(n):
    w = workloads.scatter(n, seed=n, slots=500)
    y = torch.full((n,), float("nan"), dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "gather"), idx=dev(w["idx"]), w=dev(w["w"]), table=dev(w["table"]), y=y)
    at = np.clip(w["idx"], 0, 499)
    np.testing.assert_array_equal(host(y), w["w"] * w["table"][at])


@pytest.mark.parametrize("n", SIZES)
def test_gather_vjp_scatters_into_the_table_gradient(n):
    """The adjoint of the read adds bar_y * w into bar_table[clamp(idx)] (a plain
    atomic commit) and bar_w = bar_y * table[clamp(idx)] per sample (exact)."""
    w = workloads.scatter(n, seed=n + 1, slots=500)
    bar_w = torch.full((n,), float("nan"), dtype=torch.float64, device="cuda")
    bar_table = torch.zeros(500, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "gather_vjp"), idx=dev(w["idx"]), w=dev(w["w"]), table=dev(w["table"]),
                bar_y=dev(w["bar_y"]), bar_w=bar_w, bar_table=bar_table)
    at = np.clip(w["idx"], 0, 499)
    np.testing.assert_array_equal(host(bar_w), w["bar_y"] * w["table"][at])
    want, mag, cnt = exact(at, w["bar_y"] * w["w"], 500)
    within(host(bar_table), want, mag, cnt.max() + 8)


@pytest.mark.parametrize("n", SIZES)
def test_segment_sum_default_policy_folds_its_owned_companion(n):
    """Aligned runs of the sample index (one commit per warp), compensated by
    default: the companion is the runtime's, folded into the target."""
    w = workloads.scatter(n, seed=n + 2)
    slots = -(-n // SEGMENT)
    acc = torch.zeros(slots, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "segment_sum"), x=dev(w["x"]), acc=acc)
    want, mag, _cnt = exact(np.arange(n) // SEGMENT, w["x"], slots)
    within(host(acc), want, mag, 2)


def test_segment_sum_with_a_bound_companion_keeps_the_residual_apart():
    n = 20000
    w = workloads.scatter(n, seed=5)
    slots = -(-n // SEGMENT)
    acc = torch.zeros(slots, dtype=torch.float64, device="cuda")
    comp = torch.zeros(slots, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "segment_sum"), x=dev(w["x"]), acc=acc, acc_c=comp)
    want, mag, _cnt = exact(np.arange(n) // SEGMENT, w["x"], slots)
    total = np.array([math.fsum([a, c]) for a, c in zip(host(acc), host(comp))])
    within(total, want, mag, 2)


@pytest.mark.parametrize("n", SIZES)
def test_keyed_sum_over_sorted_keys(n):
    w = workloads.scatter(n, seed=n + 3, slots=700)
    acc = torch.zeros(700, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "keyed_sum"), x=dev(w["x"]), key=dev(w["sorted_key"]), acc=acc)
    want, mag, cnt = exact(w["sorted_key"], w["x"], 700)
    within(host(acc), want, mag, cnt.max() + 8)


@pytest.mark.parametrize("n", SIZES)
def test_histogram_compensated_over_any_keys_onto_prior_values(n):
    w = workloads.scatter(n, seed=n + 4, slots=300)
    prior = np.random.default_rng(n).uniform(0.0, 1.0, 300)
    acc = dev(prior.copy())
    runtime.run(runtime.load(BUNDLES, "histogram"), x=dev(w["x"]), key=dev(w["key"]), acc=acc)
    want, mag, _cnt = exact(w["key"], w["x"], 300, prior)
    within(host(acc), want, mag, 2)


@pytest.mark.parametrize("n", SIZES)
def test_bitmask_or_commit(n):
    w = workloads.scatter(n, seed=n + 5, slots=64)
    acc = torch.zeros(64, dtype=torch.uint32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "bitmask"), bits=dev(w["bits"]), key=dev(w["key"]), acc=acc)
    want = np.zeros(64, dtype=np.uint32)
    np.bitwise_or.at(want, w["key"], w["bits"])
    np.testing.assert_array_equal(host(acc), want)


def test_a_partition_commits_only_its_samples():
    n = 50000
    w = workloads.scatter(n, seed=9, slots=128)
    acc = torch.zeros(128, dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(BUNDLES, "histogram"), x=dev(w["x"]), key=dev(w["key"]), acc=acc,
                base=1000, count=30000)
    want, mag, _cnt = exact(w["key"][1000:31000], w["x"][1000:31000], 128)
    within(host(acc), want, mag, 2)


@pytest.mark.parametrize("slots", [2048, 3000, 50000])
def test_histogram_whose_target_fits_a_block_partly_or_not_at_all(slots):
    """A block commits into shared-memory copies of its targets when they fit
    its share (2048 slots: the sum and its companion both; 3000: the sum only,
    the companion's residuals go to the plane; 50000: neither) -- the same
    contract on every path."""
    n = 300000
    w = workloads.scatter(n, seed=slots, slots=slots)
    prior = np.random.default_rng(slots).uniform(0.0, 1.0, slots)
    acc = dev(prior.copy())
    runtime.run(runtime.load(BUNDLES, "histogram"), x=dev(w["x"]), key=dev(w["key"]), acc=acc)
    want, mag, _cnt = exact(w["key"], w["x"], slots, prior)
    within(host(acc), want, mag, 2)


@pytest.mark.parametrize("slots", [64, 20000])
def test_bitmask_through_a_private_copy_and_straight_to_the_plane(slots):
    n = 200000
    w = workloads.scatter(n, seed=slots + 1, slots=slots)
    acc = torch.zeros(slots, dtype=torch.uint32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "bitmask"), bits=dev(w["bits"]), key=dev(w["key"]), acc=acc)
    want = np.zeros(slots, dtype=np.uint32)
    np.bitwise_or.at(want, w["key"], w["bits"])
    np.testing.assert_array_equal(host(acc), want)


@pytest.mark.parametrize("slots", [300, 3000, 50000])
@pytest.mark.parametrize("n", [1000, 65536 + 17, 300000])
def test_compensated_sink_policy_commits_its_residuals_into_the_declared_plane(n, slots):
    """A kernel built under the compensated sink policy (a Kind,
    hawk/ext): the scatter's commit into acc is compensated, each add's
    rounding residual going to the kernel's own plane acc_c (no runtime-owned
    companion).  acc + acc_c, per slot, is the exact sum of the prior values
    and the terms within the compensated bound; acc alone carries the plain
    bound; through shared-memory copies of the targets when they fit a block
    (300 slots), partly (3000) or not at all (50000)."""
    w = workloads.scatter(n, seed=n + slots, slots=slots)
    rng = np.random.default_rng(slots)
    prior = rng.uniform(0.0, 1.0, slots)
    x = w["x"] * np.exp(rng.uniform(-20.0, 20.0, n))       # magnitudes that round away bits
    acc, acc_c = dev(prior.copy()), torch.zeros(slots, dtype=torch.float64, device="cuda")
    k = runtime.load(BUNDLES, "comp_scatter")
    runtime.run(k, x=dev(x), key=dev(w["key"]), acc=acc, acc_c=acc_c)
    want, mag, cnt = exact(w["key"], x, slots, prior)
    a, c = host(acc), host(acc_c)
    within(a + c, want, mag, 2)
    within(a, want, mag, 2 + cnt.max())
    assert np.any(c != 0.0)                                  # the residuals were committed
