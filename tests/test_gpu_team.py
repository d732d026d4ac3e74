"""Team-form linear algebra on the B200: one matrix per lane, a warp per matrix.

Kernels whose factorisation is above the one-thread cap of 32 run as the
reference's stages (hawk/ir/team.py): a copy stage into runtime-owned scratch,
a team stage (hk/team.cuh), a reader stage.  The team stage applies every
element the one-thread form's operations in the same order, so the device is
compared with the CPU oracle (that order, for any n) bit for bit; the oracle is
pinned against the reference interpreter's LAPACK results by
tests/test_oracle_golden.py.  Failing lanes (a non-positive leading minor, a
singular matrix, a zero diagonal) report the same status and zero solutions.
Sizes: 33 and 64 staged through shared memory; 128, 160 (LU) and 512
(Cholesky) worked in place in the scratch planes.  The symmetric eigensolver
at 40 is the one-thread form's Jacobi spread over the team; least squares
with 40 unknowns is the build's Householder QR (the reference's team QR is
absent), pinned by the oracle's restatement and numpy.  The tolerance the
north star states (1e-12 relative) is asserted beside the exact comparison.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from hawk_b200 import runtime, workloads  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
EPS = np.finfo(np.float64).eps


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def nan(shape, dtype=torch.float64):
    t = torch.empty(shape, dtype=dtype, device="cuda")
    if dtype == torch.int32:
        t.fill_(-7)
    else:
        t.fill_(float("nan"))
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _exact(got, want):
    np.testing.assert_array_equal(got, want)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=0)


def run_chol(n, lanes, seed, base=0, count=None):
    w = workloads.team(n, lanes, "spd", seed)
    k = runtime.load(BUNDLES, f"team_chol_{n}")
    out = {"x": nan((n, lanes)), "X": nan((n, 2, lanes)), "L": nan((n, n, lanes)), "info": nan(lanes, torch.int32)}
    runtime.run(k, A=dev(w["A"]), b=dev(w["b"]), B=dev(w["B"]), base=base, count=count, **out)
    return w, {key: host(v) for key, v in out.items()}, k


def run_lu(n, lanes, seed):
    w = workloads.team(n, lanes, "general", seed)
    k = runtime.load(BUNDLES, f"team_lu_{n}")
    out = {"x": nan((n, lanes)), "X": nan((n, 2, lanes)), "det": nan(lanes), "info": nan(lanes, torch.int32)}
    runtime.run(k, A=dev(w["A"]), b=dev(w["b"]), B=dev(w["B"]), **out)
    return w, {key: host(v) for key, v in out.items()}, k


@pytest.mark.parametrize("n,lanes", [(33, 37), (64, 21), (128, 9)])
def test_team_cholesky_is_the_oracle_bit_for_bit(n, lanes):
    w, got, k = run_chol(n, lanes, seed=100 + n)
    x, X, L, info = oracle.team_chol(w["A"], w["b"], w["B"])
    np.testing.assert_array_equal(got["info"], info)
    assert info[workloads.TEAM_BAD] == n // 2 + 1 and np.count_nonzero(info) == 1
    _exact(got["x"], x)
    _exact(got["X"], X)
    _exact(got["L"], L)
    assert not np.any(got["x"][:, workloads.TEAM_BAD]) and not np.any(got["L"][..., workloads.TEAM_BAD])
    assert k.errors() == 0


@pytest.mark.parametrize("n,lanes", [(33, 37), (64, 21), (128, 9)])
def test_team_lu_is_the_oracle_bit_for_bit(n, lanes):
    w, got, k = run_lu(n, lanes, seed=200 + n)
    x, X, det, info = oracle.team_lu(w["A"], w["b"], w["B"])
    np.testing.assert_array_equal(got["info"], info)
    assert info[workloads.TEAM_BAD] > 0 and np.count_nonzero(info) == 1
    _exact(got["x"], x)
    _exact(got["X"], X)
    _exact(got["det"], det)
    assert got["det"][workloads.TEAM_BAD] == 0.0
    assert k.errors() == 0


def test_team_chol_from_is_the_oracle_bit_for_bit():
    w = workloads.team(64, 11, "lower", 301)
    k = runtime.load(BUNDLES, "team_chol_from_64")
    out = {"x": nan((64, 11)), "L": nan((64, 64, 11)), "info": nan(11, torch.int32)}
    runtime.run(k, A=dev(w["A"]), b=dev(w["b"]), **out)
    got = {key: host(v) for key, v in out.items()}
    x, L, info = oracle.team_chol_from(w["A"], w["b"])
    np.testing.assert_array_equal(got["info"], info)
    assert info[workloads.TEAM_BAD] == 1
    _exact(got["x"], x)
    _exact(got["L"], L)


def test_a_matrix_of_512_is_worked_in_its_scratch_plane():
    """Cholesky at 512 (2 MB a matrix, beyond a block's shared memory): the team
    works the lane's scratch slice in place; same bits as the oracle."""
    n, lanes = 512, 5
    w = workloads.team(n, lanes, "spd", 512)
    k = runtime.load(BUNDLES, "team_chol_512")
    out = {"x": nan((n, lanes)), "info": nan(lanes, torch.int32)}
    runtime.run(k, A=dev(w["A"]), b=dev(w["b"]), **out)
    got = {key: host(v) for key, v in out.items()}
    x, _X, _L, info = oracle.team_chol(w["A"], w["b"], np.zeros((n, 2, lanes)))
    np.testing.assert_array_equal(got["info"], info)
    _exact(got["x"], x)
    a = np.moveaxis(w["A"], -1, 0)
    for lane in (0, 1, 3, 4):
        r = np.abs(a[lane] @ got["x"][:, lane] - w["b"][:, lane]).max()
        assert r / (n * EPS * (np.abs(a[lane]).max() * np.abs(got["x"][:, lane]).max())) < 50


def test_lu_at_160_is_worked_in_its_scratch_plane():
    n, lanes = 160, 6
    w = workloads.team(n, lanes, "general", 160)
    k = runtime.load(BUNDLES, "team_lu_160")
    out = {"x": nan((n, lanes)), "det": nan(lanes), "info": nan(lanes, torch.int32)}
    runtime.run(k, A=dev(w["A"]), b=dev(w["b"]), **out)
    got = {key: host(v) for key, v in out.items()}
    x, _X, det, info = oracle.team_lu(w["A"], w["b"], np.zeros((n, 2, lanes)))
    np.testing.assert_array_equal(got["info"], info)
    _exact(got["x"], x)
    _exact(got["det"], det)


def test_a_partition_runs_only_its_lanes():
    """base/count: the lanes outside the partition keep what the planes held."""
    n, lanes = 33, 12
    w, got, _k = run_chol(n, lanes, seed=7, base=3, count=6)
    x, _X, _L, info = oracle.team_chol(w["A"], w["b"], w["B"])
    _exact(got["x"][:, 3:9], x[:, 3:9])
    np.testing.assert_array_equal(got["info"][3:9], info[3:9])
    assert np.isnan(got["x"][:, :3]).all() and np.isnan(got["x"][:, 9:]).all()
    assert (got["info"][:3] == -7).all() and (got["info"][9:] == -7).all()


def test_two_runs_in_a_row_and_a_single_lane():
    """The scratch planes the runtime owns are reused run to run; one lane runs too."""
    n = 64
    for lanes, seed in ((1, 11), (5, 12), (5, 13)):
        w, got, _k = run_chol(n, lanes, seed=seed)
        x, X, L, info = oracle.team_chol(w["A"], w["b"], w["B"])
        _exact(got["x"], x)
        _exact(got["L"], L)
        np.testing.assert_array_equal(got["info"], info)


def test_team_eigh_is_the_one_thread_order_bit_for_bit():
    """eigh at n = 40 (a team stage): the one-thread form's cyclic Jacobi with
    each rotation's updates spread over the team -- the oracle's bits, the
    repeated eigenvalue of lane 2 reported in bit 2."""
    n, lanes = 40, 7
    rng = np.random.default_rng(40)
    mats = []
    for lane in range(lanes):
        g = rng.standard_normal((n, n))
        a = (g + g.T) / 2
        if lane == 2:
            q, _ = np.linalg.qr(rng.standard_normal((n, n)))
            a = (q * np.r_[np.ones(n // 2), np.linspace(2, 3, n - n // 2)]) @ q.T
        mats.append(a)
    A = np.ascontiguousarray(np.moveaxis(np.stack(mats), 0, -1))
    k = runtime.load(BUNDLES, "team_eigh_40")
    out = {"w": nan((n, lanes)), "V": nan((n, n, lanes)), "info": nan(lanes, torch.int32)}
    runtime.run(k, A=dev(A), **out)
    got = {key: host(v) for key, v in out.items()}
    w, V, info = oracle.sym_eigen(A)
    np.testing.assert_array_equal(got["info"], info)
    _exact(got["w"], w)
    _exact(got["V"], V)
    assert info[2] & 2
    for lane in (0, 1, 3):
        np.testing.assert_allclose(got["w"][:, lane], np.linalg.eigvalsh(mats[lane]), rtol=0,
                                   atol=100 * n * EPS * np.abs(mats[lane]).max() * n)


def test_team_lstsq_by_householder_qr():
    """lstsq(J, r) with 40 unknowns (80 x 40 J): the team-form Householder QR
    and its solve -- the oracle's bits; a zero column reports info 2 (the first
    zero diagonal of R) and a zero solution; the rest within the reference's
    bound of numpy's least squares (50 n eps cond |x|)."""
    m_rows, n, lanes = 80, 40, 5
    rng = np.random.default_rng(80)
    J = rng.standard_normal((lanes, m_rows, n))
    r = rng.standard_normal((lanes, m_rows))
    J[2, :, 1] = 0.0
    Jp = np.ascontiguousarray(np.moveaxis(J, 0, -1))
    rp = np.ascontiguousarray(r.T)
    k = runtime.load(BUNDLES, "team_lstsq_40")
    out = {"x": nan((n, lanes)), "info": nan(lanes, torch.int32)}
    runtime.run(k, J=dev(Jp), r=dev(rp), **out)
    got = {key: host(v) for key, v in out.items()}
    x, info = oracle.lstsq_qr(Jp, rp)
    np.testing.assert_array_equal(got["info"], info)
    _exact(got["x"], x)
    assert info[2] == 2 and not np.any(got["x"][:, 2])
    for lane in (0, 1, 3, 4):
        want = np.linalg.lstsq(J[lane], r[lane], rcond=None)[0]
        cond = np.linalg.cond(J[lane])
        assert np.abs(got["x"][:, lane] - want).max() <= 50 * n * EPS * cond * np.abs(want).max()


@pytest.mark.parametrize("mode", ["float64", "float32"])
def test_warp_form_eigenvalues_at_32(mode):
    """An eigenvalues-only 32 x 32 eigh takes the reference's warp entry on a
    device-only sm_100 build (hawk/ir/team.py:236-275): a copy stage, an
    eigh_warp stage (one warp a lane, hk::linalg::warp::eighValues), a reader.
    In float64 its values and status are the one-thread form's bits (the
    oracle's); in float32 within the one-thread form's rounding of numpy's
    float64 eigenvalues, and the repeated eigenvalue of lane 2 reported in bit 2."""
    n, lanes = 32, 9
    rng = np.random.default_rng(32)
    mats = []
    for lane in range(lanes):
        g = rng.standard_normal((n, n))
        a = (g + g.T) / 2
        if lane == 2:
            q, _ = np.linalg.qr(rng.standard_normal((n, n)))
            a = (q * np.r_[np.ones(n // 2), np.linspace(2, 3, n - n // 2)]) @ q.T
        mats.append(a)
    dt = np.float64 if mode == "float64" else np.float32
    A = np.ascontiguousarray(np.moveaxis(np.stack(mats), 0, -1)).astype(dt)
    k = runtime.load(BUNDLES, "warp_eigvals_32", mode)
    w = torch.full((n, lanes), float("nan"), dtype=torch.float64 if mode == "float64" else torch.float32,
                   device="cuda")
    info = nan(lanes, torch.int32)
    runtime.run(k, A=dev(A), w=w, info=info)
    got_w, got_info = host(w), host(info)
    assert got_info[2] & 2
    if mode == "float64":
        want_w, _v, want_info = oracle.sym_eigen(A, vectors=False)
        np.testing.assert_array_equal(got_info, want_info)
        _exact(got_w, want_w)
    else:
        eps32 = np.finfo(np.float32).eps
        for lane in range(lanes):
            ref = np.linalg.eigvalsh(A[..., lane].astype(np.float64))
            bound = 100 * n * eps32 * np.abs(A[..., lane]).max() * n
            np.testing.assert_allclose(got_w[:, lane], ref, rtol=0, atol=bound)
