"""Automatic stepping kernels on the B200: the fused entry and the persistent entry.

An automatic kernel (steps="auto", hawk/trace/steps.py) runs, per launch and
per sample not finished on entry, the single step (fused_steps word 1) or up to
``word`` trips of its fused loop, leaving at its finish; the finished counter
counts the samples newly finished (hawk/emit/wrapper.py:1507-1545).  The
persistent entry (hawk/emit/cuda.py:464-707 is the reference's) runs every
sample exactly as one fused launch with the same word would, from lanes that
claim samples off a counter; its finished counter holds the batch's finished
count (on entry included), ``hawk_steps`` the longest per-sample trip count,
``hawk_stepsum`` and ``hawk_util[0]`` the trips run.

Checked against the oracle bit for bit (the kernels use only correctly rounded
operations: + - * /, sqrt, fmin/fmax), at the reference's ragged sizes, with
samples finished on entry, for words 1, 0, a negative one, and budgets that
cut samples mid-run; the persistent entry for chunks 1, 3, 32 and 0 (whole
samples) on the default grid and a grid of one block.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from hawk_b200 import runtime, workloads  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
SIZES = [1, 33, 1000, 65536 + 17]


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def word_of(w):
    return torch.tensor([w], dtype=torch.int64, device="cuda")


def counter():
    return torch.zeros(1, dtype=torch.uint32, device="cuda")


OSC = ("x", "v", "k", "nstop", "omega", "zeta", "terminated")
ORB = ("s", "t", "h", "n_acc", "n_rej", "t_end", "terminated")


def osc_workload(n, seed=0, stop_max=40):
    return workloads.oscillator(n, seed=seed, stop_max=stop_max, done_every=7)


def orb_workload(n, seed=0):
    return workloads.orbit(n, seed=seed, done_every=7)


def to_dev(w, names):
    return {k: dev(w[k]) for k in names}


def oracle_planes(w, names):
    return {k: np.array(w[k], copy=True) for k in names}


def same_planes(got: dict, want: dict, names):
    for k in names:
        g, e = host(got[k]), want[k]
        assert np.array_equal(g, e, equal_nan=True), (k, np.flatnonzero(g != e)[:5])


# ----------------------------------------------------------------- fused entry
@pytest.mark.parametrize("word", [1, 0, -2, 5, 64])
@pytest.mark.parametrize("n", SIZES)
def test_oscillator_fused_entry_matches_the_oracle(n, word):
    w = osc_workload(n, seed=n)
    planes, want = to_dev(w, OSC), oracle_planes(w, OSC)
    fin = counter()
    runtime.run(runtime.load(BUNDLES, "oscillator"), **planes, dt=w["dt"], fused_steps=word_of(word),
                finished_count=fin)
    want_fin = oracle.oscillator(want, w["dt"], word)
    same_planes(planes, want, OSC)
    assert int(host(fin)[0]) == want_fin


@pytest.mark.parametrize("word", [1, 9, 64])
@pytest.mark.parametrize("n", [1, 33, 1000, 20000])
def test_orbit_fused_entry_matches_the_oracle(n, word):
    w = orb_workload(n, seed=n)
    planes, want = to_dev(w, ORB), oracle_planes(w, ORB)
    fin = counter()
    runtime.run(runtime.load(BUNDLES, "orbit"), **planes, fused_steps=word_of(word), finished_count=fin)
    want_fin = oracle.orbit(want, word, threads=8)
    same_planes(planes, want, ORB)
    assert int(host(fin)[0]) == want_fin
    if word == 64 and n >= 1000:
        assert want["n_rej"].sum() > 0 and want_fin > 0


def test_a_run_without_the_reserved_words_takes_one_step():
    """Left out, the word is 1 and the counter a fresh zero the kernel keeps
    (hawk/runtime.py:237-265)."""
    n = 4096
    w = osc_workload(n, seed=3, stop_max=2)
    planes, want = to_dev(w, OSC), oracle_planes(w, OSC)
    k = runtime.load(BUNDLES, "oscillator")
    for _ in range(2):
        runtime.run(k, **planes, dt=w["dt"])
        want_fin = oracle.oscillator(want, w["dt"], 1)
        same_planes(planes, want, OSC)
        assert int(host(k.finished)[0]) == want_fin


def test_a_runner_loop_finishes_every_sample():
    """Fused launches of 16 steps until the counters add up to every sample
    not finished on entry: the same planes as the oracle's same launches."""
    n = 30000
    w = osc_workload(n, seed=11, stop_max=100)
    planes, want = to_dev(w, OSC), oracle_planes(w, OSC)
    k = runtime.load(BUNDLES, "oscillator")
    todo = int((~w["terminated"]).sum())
    done, launches = 0, 0
    while done < todo:
        fin = counter()
        runtime.run(k, **planes, dt=w["dt"], fused_steps=word_of(16), finished_count=fin)
        got = int(host(fin)[0])
        assert got == oracle.oscillator(want, w["dt"], 16)
        done += got
        launches += 1
        assert launches <= 7
    same_planes(planes, want, OSC)
    assert host(planes["terminated"]).all()


# ------------------------------------------------------------ persistent entry
def trips_of(name, before, after):
    if name == "oscillator":
        return after["k"] - before["k"]
    return (after["n_acc"] + after["n_rej"]) - (before["n_acc"] + before["n_rej"])


@pytest.mark.parametrize("grid", [0, 1])
@pytest.mark.parametrize("chunk", [1, 3, 32, 0])
@pytest.mark.parametrize("name,word", [("oscillator", 1000), ("oscillator", 13), ("orbit", 1000), ("orbit", 9)])
def test_persistent_entry_is_one_fused_launch(name, word, chunk, grid):
    n = 20000 if name == "oscillator" else 3000
    w = osc_workload(n, seed=5) if name == "oscillator" else orb_workload(n, seed=5)
    names = OSC if name == "oscillator" else ORB
    extra = {"dt": w["dt"]} if name == "oscillator" else {}
    k = runtime.load(BUNDLES, name)
    fused, pers = to_dev(w, names), to_dev(w, names)
    runtime.run(k, **fused, **extra, fused_steps=word_of(word), finished_count=counter())
    steps = torch.zeros(1, dtype=torch.uint32, device="cuda")
    stepsum = torch.zeros(1, dtype=torch.uint64, device="cuda")
    util = torch.zeros(2, dtype=torch.uint64, device="cuda")
    fin = counter()
    claim = runtime.run_persist(k, **pers, **extra, fused_steps=word_of(word), finished_count=fin, chunk=chunk,
                                grid=grid, steps=steps, stepsum=stepsum, util=util)
    same_planes(pers, {key: host(v) for key, v in fused.items()}, names)
    before = {key: np.asarray(w[key]) for key in names}
    after = {key: host(v) for key, v in pers.items()}
    trips = trips_of(name, before, after)
    assert int(host(fin)[0]) == int(after["terminated"].sum())          # the batch's finished count
    assert int(host(steps)[0]) == int(trips.max())
    assert int(host(stepsum)[0]) == int(trips.sum()) == int(host(util)[0])
    assert int(host(util)[1]) >= int(host(util)[0])                     # lane slots offered >= steps run
    assert int(host(claim)[0]) >= n


def test_persistent_entry_with_no_budget_writes_back_unchanged():
    n = 5000
    w = osc_workload(n, seed=2)
    k = runtime.load(BUNDLES, "oscillator")
    for word in (0, -5):
        planes = to_dev(w, OSC)
        fin = counter()
        runtime.run_persist(k, **planes, dt=w["dt"], fused_steps=word_of(word), finished_count=fin)
        same_planes(planes, oracle_planes(w, OSC), OSC)
        assert int(host(fin)[0]) == int(w["terminated"].sum())


def test_persistent_entry_refusals():
    from hawk_b200.errors import HawkError

    with pytest.raises(HawkError, match="no persistent entry"):
        runtime.run_persist(runtime.load(BUNDLES, "energy"), v=dev(np.zeros((3, 4))), out=dev(np.zeros(4)))
    w = osc_workload(64)
    with pytest.raises(HawkError, match="steps="):
        runtime.run_persist(runtime.load(BUNDLES, "oscillator"), **to_dev(w, OSC), dt=w["dt"],
                            steps=torch.zeros(1, dtype=torch.int64, device="cuda"))


# ----------------------------------------------------------------- range entry
@pytest.mark.parametrize("name,word", [("oscillator", 1), ("oscillator", 1000), ("oscillator", 13), ("oscillator", 0),
                                       ("orbit", 1), ("orbit", 1000), ("orbit", 9)])
def test_range_entry_is_one_fused_launch_and_reports_its_steps(name, word):
    """<name>_range (hawk/emit/cuda.py:709-784 is the reference's): the bits of
    one launch of the kernel's own entry with the same word; the finished
    counter the batch's finished count (on entry included); hawk_steps the
    longest per-sample step count, hawk_stepsum the steps run."""
    n = 20000 + 17 if name == "oscillator" else 3000 + 5
    w = osc_workload(n, seed=9) if name == "oscillator" else orb_workload(n, seed=9)
    names = OSC if name == "oscillator" else ORB
    extra = {"dt": w["dt"]} if name == "oscillator" else {}
    k = runtime.load(BUNDLES, name)
    fused, ranged = to_dev(w, names), to_dev(w, names)
    runtime.run(k, **fused, **extra, fused_steps=word_of(word), finished_count=counter())
    steps = torch.zeros(1, dtype=torch.uint32, device="cuda")
    stepsum = torch.zeros(1, dtype=torch.uint64, device="cuda")
    fin = counter()
    runtime.run_range(k, **ranged, **extra, fused_steps=word_of(word), finished_count=fin, steps=steps,
                      stepsum=stepsum)
    same_planes(ranged, {key: host(v) for key, v in fused.items()}, names)
    before = {key: np.asarray(w[key]) for key in names}
    after = {key: host(v) for key, v in ranged.items()}
    trips = trips_of(name, before, after)
    assert int(host(fin)[0]) == int(after["terminated"].sum())
    assert int(host(steps)[0]) == int(trips.max())
    assert int(host(stepsum)[0]) == int(trips.sum())
    if word == 1:
        assert set(np.unique(trips)) <= {0, 1}


def test_range_entry_runs_its_partition_only_and_reports_nothing_when_asked_nothing():
    n = 5000
    w = osc_workload(n, seed=4)
    k = runtime.load(BUNDLES, "oscillator")
    planes = to_dev(w, OSC)
    runtime.run_range(k, **planes, dt=w["dt"], fused_steps=word_of(1000), finished_count=counter(),
                      base=1000, count=2000)
    want = oracle_planes(w, OSC)
    oracle.oscillator(want, w["dt"], 1000)
    got = {key: host(v) for key, v in planes.items()}
    for key in OSC:
        assert np.array_equal(got[key][1000:3000], want[key][1000:3000], equal_nan=True), key
        assert np.array_equal(got[key][:1000], np.asarray(w[key])[:1000], equal_nan=True), key
        assert np.array_equal(got[key][3000:], np.asarray(w[key])[3000:], equal_nan=True), key


def test_range_entry_refusals():
    from hawk_b200.errors import HawkError

    with pytest.raises(HawkError, match="no range entry"):
        runtime.run_range(runtime.load(BUNDLES, "energy"), v=dev(np.zeros((3, 4))), out=dev(np.zeros(4)))
    w = osc_workload(64)
    with pytest.raises(HawkError, match="stepsum="):
        runtime.run_range(runtime.load(BUNDLES, "oscillator"), **to_dev(w, OSC), dt=w["dt"],
                          stepsum=torch.zeros(1, dtype=torch.uint32, device="cuda"))
