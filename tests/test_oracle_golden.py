"""The CPU oracle against the reference's own answers.

Golden vectors come from the reference's numpy IR interpreter evaluating the
traced kernels (tests/golden/make_golden.py); the ordered-finish fixtures from
the reference's ``hawk._cells.finish``; the known answers from the reference's
README (energy) and a Kepler root.  Tolerances: 1e-12 relative for float64
values (the interpreter's numpy/LAPACK order differs from the host unit's),
exact for integer planes and for the finish tree (same operations, same order).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle

RTOL = 1e-12


def close(got, want, rtol=RTOL, atol=0.0):
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


def test_energy_known_answer():
    # README.md:80-99 of the reference: energy of these four samples and its gradient
    v = np.array([[1.0, 2.0, 3.0, 4.0], [0.0, 1.0, 0.0, 1.0], [0.0, 0.0, 1.0, 1.0]])
    np.testing.assert_array_equal(oracle.energy(v), [0.5, 2.5, 5.0, 9.0])
    np.testing.assert_array_equal(oracle.energy_vjp(v, np.ones(4)), v)


def test_energy_golden(golden):
    g = golden("energy")
    close(oracle.energy(g["v"]), g["out"])
    close(oracle.energy_vjp(g["v"], g["bar_out"]), g["bar_v"])
    close(oracle.energy_jvp(g["v"], g["dot_v"]), g["dot_out"])


def test_poly_loss_golden(golden):
    g = golden("poly_loss")
    close(oracle.poly_loss(g["x"], g["t"], float(g["a"]), float(g["b"]), float(g["c"])), g["r"])


def test_poly_loss_rows_are_per_32_sums_of_the_gradient_terms(golden):
    # hawk tests/test_sample_sum.py:38, :96-123: rows equal the float64 per-32
    # sums within 1e-14 of the row's sum of |term|
    g = golden("poly_loss")
    hi, comp = oracle.poly_loss_vjp_rows(g["x"], g["t"], g["bar_r"], float(g["a"]), float(g["b"]), float(g["c"]))
    n = g["x"].shape[0]
    for k, name in enumerate(("term_a", "term_b", "term_c")):
        terms = g[name]
        for j in range(hi.shape[1]):
            seg = terms[32 * j:min(32 * j + 32, n)]
            want = float(np.sum(seg.astype(np.longdouble)))
            assert abs((hi[k, j] + comp[k, j]) - want) <= 1e-14 * float(np.sum(np.abs(seg))) + 1e-300


def test_poly_loss_param_gradients_are_the_sums_of_the_terms(golden):
    g = golden("poly_loss")
    cells, _ = oracle.poly_loss_vjp(g["x"], g["t"], g["bar_r"], float(g["a"]), float(g["b"]), float(g["c"]))
    for k, name in enumerate(("term_a", "term_b", "term_c")):
        want = float(np.sum(g[name].astype(np.longdouble)))
        assert abs(cells[k] - want) <= 1e-14 * float(np.sum(np.abs(g[name])))


@pytest.mark.parametrize("n", [1, 2, 31, 255, 256, 257, 4095, 4096, 4097, 12289, 16385])
def test_cells_finish_is_the_reference_tree_bit_for_bit(golden, n):
    g = golden("cells")
    hi, comp = g[f"hi_{n}"], g[f"comp_{n}"]
    for op in ("sum", "max", "min"):
        got = oracle.cells_finish(hi, comp if op == "sum" else None, op)
        assert got == float(g[f"{op}_{n}"]), (op, n)
    got32 = oracle.cells_finish(hi.astype(np.float32), comp.astype(np.float32), "sum")
    assert np.float32(got32) == g[f"sum32_{n}"]


def test_gravity_golden(golden):
    g = golden("gravity")
    f, u = oracle.gravity(g["r1"], g["r2"], g["m1"], g["m2"], float(g["G"]))
    close(f, g["f"])
    close(u, g["u"])
    # measured worst relative differences from the interpreter: 3.9e-15 (JVP),
    # 8.3e-16 (VJP) -- its numpy expression order, not the host unit's
    df, du = oracle.gravity_jvp(g["r1"], g["r2"], g["dr1"], g["dr2"], g["m1"], g["m2"], float(g["G"]))
    close(df, g["dot_f"])
    close(du, g["dot_u"])
    b1, b2 = oracle.gravity_vjp(g["r1"], g["r2"], g["bar_f"], g["bar_u"], g["m1"], g["m2"], float(g["G"]))
    close(b1, g["bar_r1"])
    close(b2, g["bar_r2"])


def test_spd_solve_golden(golden):
    g = golden("spd_solve")
    close(oracle.spd_solve(g["A"], g["b"]), g["x"])
    bar_A, bar_b = oracle.spd_solve_vjp(g["A"], g["b"], g["bar_x"])
    close(bar_b, g["bar_b"])
    close(bar_A, g["bar_A"])


def test_kepler_golden(golden):
    g = golden("kepler")
    E, it = oracle.kepler(g["e"], g["M"])
    close(E, g["E"])
    np.testing.assert_array_equal(it, g["iters"])
    # glibc's sin/cos on both sides: measured bit-identical to the interpreter
    be, bM = oracle.kepler_vjp(g["e"], g["M"], g["bar_E"])
    close(be, g["bar_e"])
    close(bM, g["bar_M"])


def test_kepler_known_answer(golden):
    g = golden("kepler")
    E, it = oracle.kepler(np.array([0.5]), np.array([1.0]))
    assert E[0] == float(g["known_E"]) == 1.4987011335178484
    assert it[0] == int(g["known_iters"]) == 6


def test_a_planted_fault_in_the_oracle_is_caught(golden):
    # non-vacuity (the reference's tests/test_serial_oracle.py:33-48 plants one too):
    # a perturbed input must move the output beyond the tolerance used above
    g = golden("energy")
    v = g["v"].copy()
    v[0, 5] *= 1.0 + 1e-9
    with pytest.raises(AssertionError):
        close(oracle.energy(v), g["out"])


OSC_WORDS = (1, 0, -2, 5, 30)
ORB_WORDS = (1, 9, 40)


@pytest.mark.parametrize("word", OSC_WORDS)
def test_oscillator_golden(golden, word):
    """The automatic RK4 oscillator, one launch with each fused_steps word, against
    the interpreter's single step (word 1) and fused loop: bit-identical (the
    same operations in the same order), finished samples marked and counted."""
    g = golden("steps")
    planes = {k: np.array(g[f"osc_{k}"], copy=True) for k in ("x", "v", "k", "nstop", "omega", "zeta")}
    planes["terminated"] = np.zeros(planes["x"].shape[0], dtype=bool)
    fin = oracle.oscillator(planes, float(g["osc_dt"]), word)
    for k in ("x", "v", "k"):
        np.testing.assert_array_equal(planes[k], g[f"osc_w{word}_{k}"])
    want_term = g[f"osc_w{word}_terminated"].astype(bool)
    np.testing.assert_array_equal(planes["terminated"], want_term)
    assert fin == int(want_term.sum())


@pytest.mark.parametrize("word", ORB_WORDS)
def test_orbit_golden(golden, word):
    """The automatic Fehlberg 7(8) orbit kernel (accepted and rejected attempts,
    samples finishing at their final time) against the interpreter: bit-identical."""
    g = golden("steps")
    planes = {k: np.array(g[f"orb_{k}"], copy=True) for k in ("s", "t", "h", "n_acc", "n_rej", "t_end")}
    planes["terminated"] = np.zeros(planes["t"].shape[0], dtype=bool)
    fin = oracle.orbit(planes, word)
    for k in ("s", "t", "h", "n_acc", "n_rej"):
        np.testing.assert_array_equal(planes[k], g[f"orb_w{word}_{k}"])
    want_term = g[f"orb_w{word}_terminated"].astype(bool)
    np.testing.assert_array_equal(planes["terminated"], want_term)
    assert fin == int(want_term.sum())
    if word == 40:
        assert planes["n_rej"].sum() > 0 and fin > 0          # the fixture exercises rejects and finishes


def test_stepping_samples_finished_on_entry_are_left_alone(golden):
    """A sample finished on entry is skipped: no plane moves and it is not counted."""
    g = golden("steps")
    planes = {k: np.array(g[f"osc_{k}"], copy=True) for k in ("x", "v", "k", "nstop", "omega", "zeta")}
    n = planes["x"].shape[0]
    planes["terminated"] = (np.arange(n) % 5) == 2
    before = {k: planes[k].copy() for k in ("x", "v", "k")}
    fin = oracle.oscillator(planes, float(g["osc_dt"]), 30)
    skip = (np.arange(n) % 5) == 2
    for k in ("x", "v", "k"):
        np.testing.assert_array_equal(planes[k][skip], before[k][skip])
        np.testing.assert_array_equal(planes[k][~skip], g[f"osc_w30_{k}"][~skip])
    assert fin == int(g["osc_w30_terminated"].astype(bool)[~skip].sum())


EPS = np.finfo(np.float64).eps


def _team(g, name):
    return {k[len(name) + 1:]: v for k, v in g.items() if k.startswith(name + "_")}


@pytest.mark.parametrize("name", ["team_chol_33", "team_chol_64"])
def test_team_cholesky_golden(golden, name):
    """The team-form Cholesky kernel against the interpreter (scipy LAPACK):
    the status exactly, the factor within 50 n eps |A|, the solves to the
    interpreter's within 1e-10 relative (the tolerances of the reference's
    tests/test_team_linalg.py)."""
    g = _team(golden("team"), name)
    n = g["A"].shape[0]
    x, X, L, info = oracle.team_chol(g["A"], g["b"], g["B"])
    np.testing.assert_array_equal(info, g["info"])
    scale = np.abs(g["A"]).max()
    assert np.abs(L - g["L"]).max() <= 50 * n * EPS * scale
    close(x, g["x"], rtol=1e-10, atol=1e-13)
    close(X, g["X"], rtol=1e-10, atol=1e-13)
    bad = np.flatnonzero(info)
    assert bad.tolist() == [2] and info[2] == n // 2 + 1
    assert not np.any(x[:, 2]) and not np.any(X[..., 2]) and not np.any(L[..., 2])


def test_team_lu_golden(golden):
    g = _team(golden("team"), "team_lu_33")
    x, X, det, info = oracle.team_lu(g["A"], g["b"], g["B"])
    np.testing.assert_array_equal(info, g["info"])
    assert info[2] > 0 and not np.any(x[:, 2]) and det[2] == 0.0
    close(x, g["x"], rtol=1e-10, atol=1e-13)
    close(X, g["X"], rtol=1e-10, atol=1e-13)
    close(det, g["det"], rtol=1e-9 * 33)


def test_team_chol_from_golden(golden):
    g = _team(golden("team"), "team_chol_from_64")
    x, L, info = oracle.team_chol_from(g["A"], g["b"])
    np.testing.assert_array_equal(info, g["info"])
    np.testing.assert_array_equal(L, g["L"])
    close(x, g["x"], rtol=1e-10, atol=1e-13)
    assert info[2] == 1 and not np.any(x[:, 2])


def test_read_back_sums_match_numpy():
    """The oracle's read-back kernels (rows + ordered finish, then the reading
    bodies) against numpy with exact sums (math.fsum): within the reference's
    sample-sum tolerance, 1e-14 relative to the sum of magnitudes
    (tests/test_sample_sum.py:38 of the reference)."""
    import math

    rng = np.random.default_rng(7)
    for n in (1, 33, 5000, 270000):
        x = rng.uniform(0.5, 1.5, n)
        s = math.fsum(x)
        close(oracle.share(x), x / s, rtol=1e-14)
        y = rng.normal(3.0, 2.0, n)
        mu, z, t = oracle.standard(y)
        want_mu = math.fsum(y / n)
        assert abs(mu - want_mu) <= 1e-14 * math.fsum(np.abs(y / n))
        if n > 1:
            d = y - want_mu
            v = math.fsum(d * d / n)
            close(z, d / math.sqrt(v), rtol=1e-12)
            assert abs(t - math.fsum(z * z)) <= 1e-14 * math.fsum(z * z)
        v3 = np.stack([x, x * x, 2 * x])
        want = v3 - np.array([math.fsum(v3[k] / n) for k in range(3)])[:, None]
        close(oracle.centred(x), want, rtol=1e-12, atol=1e-15)


def test_sample_sum_max_and_min_ignore_nan():
    x = np.array([1.0, np.nan, 3.0, -2.0] * 20)
    assert oracle.sample_sum(x, "max") == 3.0
    assert oracle.sample_sum(x, "min") == -2.0


def test_key_sums_match_exact_sums():
    import math

    x = np.random.default_rng(3).normal(0.0, 1.0, 8 * 500)
    got = oracle.key_sums(x)
    for k in range(500):
        seg = x[8 * k:8 * k + 8]
        assert abs(got[k] - math.fsum(seg)) <= 8 * np.finfo(float).eps * math.fsum(np.abs(seg))
    close(oracle.key_share(np.ones(16)), np.full(16, 1 / 8.0))


def test_block_sums_match_numpy():
    rng = np.random.default_rng(11)
    j = rng.normal(0.0, 1.0, (6, 8 * 50))
    got = oracle.block_sums(j, j)
    jj = j.reshape(6, 50, 8)
    close(got, np.einsum("akr,bkr->abk", jj, jj), rtol=1e-13, atol=1e-13)
    close(oracle.block_sums(j), jj.sum(axis=2), rtol=1e-13, atol=1e-13)


def test_eigh_golden(golden):
    """Cyclic Jacobi (the oracle) against numpy's eigh through the reference
    interpreter: the status exactly (bit 2 marks the repeated eigenvalue), the
    values and vectors within the reference's tests/test_team_linalg.py bounds
    (100 n eps |A| n), the vectors orthonormal and signed alike."""
    g = golden("eigen")
    w, V, info = oracle.sym_eigen(g["A"])
    np.testing.assert_array_equal(info & 2, g["info"] & 2)
    assert (info & 1 == 0).all() and info[2] & 2
    n = g["A"].shape[0]
    for lane in range(g["A"].shape[-1]):
        s = g["A"][..., lane]
        tol = 100 * n * EPS * np.abs(s).max() * n
        np.testing.assert_allclose(w[:, lane], g["w"][:, lane], rtol=0, atol=tol)
        v = V[..., lane]
        np.testing.assert_allclose(s @ v, v * w[:, lane], rtol=0, atol=tol)
        np.testing.assert_allclose(v.T @ v, np.eye(n), rtol=0, atol=100 * n * EPS)
        if lane != 2:           # a repeated eigenvalue's vectors are any basis of its space
            np.testing.assert_allclose(v, g["V"][..., lane], rtol=0, atol=1e-9)


def test_lstsq_qr_matches_numpy():
    rng = np.random.default_rng(5)
    J = rng.standard_normal((80, 40, 3))
    r = rng.standard_normal((80, 3))
    x, info = oracle.lstsq_qr(np.ascontiguousarray(J), np.ascontiguousarray(r))
    assert (info == 0).all()
    for lane in range(3):
        want = np.linalg.lstsq(J[..., lane], r[:, lane], rcond=None)[0]
        cond = np.linalg.cond(J[..., lane])
        assert np.abs(x[:, lane] - want).max() <= 50 * 40 * EPS * cond * np.abs(want).max()


def ordered_draw(rows: int, keys: int) -> np.ndarray:
    """The lanes of an ordered-sum fixture, drawn as tests/golden/make_golden.py draws them."""
    n = rows * keys
    return np.random.default_rng(n).normal(size=n) * np.exp(np.random.default_rng(n + 1).normal(size=n))


@pytest.mark.parametrize("rows,keys", [(8, 5), (1, 3), (1000, 2), (65536, 1), (197385, 2), (200003, 1)])
def test_ordered_sums_are_the_reference_fixed_tree_bitwise(golden, rows, keys):
    """Every key's ordered sum equals the reference's numpy emulation of the
    fixed grouping (its tests/test_ordered_fixed_tree.py:33-40) bit for bit:
    a partial block, a key of one lane, exactly one stride, three strides."""
    import hashlib

    g = golden("ordered")
    x = ordered_draw(rows, keys)
    assert hashlib.sha256(x.tobytes()).digest() == g[f"sha_{rows}_{keys}"].tobytes()
    np.testing.assert_array_equal(oracle.ordered_sums(x, rows), g[f"sum_{rows}_{keys}"])


def test_scatter_chunks_are_the_reference_choice():
    """clamp(n // cells, 1, 256): the reference's known answers
    (tests/test_scatter_ordered.py:119-121 there)."""
    from hawk_b200.runtime import SplitKernel

    cases = ((20000, 7), (50, 200), (1000, 1000), (10**6, 10**4), (10**6, 1), (10, 0))
    assert [SplitKernel.scatter_chunks(n, t) for n, t in cases] == [256, 1, 1, 100, 256, 10]


@pytest.mark.parametrize("n,cells,heavy", [(20000, 7, True), (3000, 1, False), (5000, 40, False),
                                           (50, 200, False), (1000, 1000, False), (30000, 1500, False)])
def test_ordered_scatter_is_add_at_within_the_reference_bound(n, cells, heavy):
    """The chunked walk adds what np.add.at adds (the reference's bound:
    1e-12 relative to the largest cell), skips key -1, and an empty cell
    stays exactly 0; onto a plane that held values it adds on top."""
    rng = np.random.default_rng(n)
    key = rng.integers(0, cells, n).astype(np.int32)
    if heavy:
        key[rng.random(n) < 0.9] = cells // 2
    if cells == 40:
        key[key == 13] = 14
    key[::7] = -1
    x = rng.normal(size=n) * np.exp(rng.normal(size=n))
    got, bad = oracle.ordered_scatter(key, x, np.zeros(cells))
    assert not bad
    want = np.zeros(cells)
    np.add.at(want, key[key >= 0], x[key >= 0])
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12 * np.abs(want).max(initial=1.0))
    if cells == 40:
        assert got[13] == 0.0
    base = np.linspace(1.0, 2.0, cells)
    more, _ = oracle.ordered_scatter(key, x, base)
    np.testing.assert_array_equal(more, base + got)


def test_ordered_scatter_reports_a_key_out_of_range():
    key = np.zeros(300, np.int32)
    x = np.ones(300)
    for bad in (9, 14, -2, 2**31 - 2):
        wild = key.copy()
        wild[[3, 299]] = bad
        got, flagged = oracle.ordered_scatter(wild, x, np.zeros(9))
        assert flagged and got[0] == 298.0
    assert oracle.ordered_scatter(np.full(300, -1, np.int32), x, np.zeros(0))[1] is False
    assert oracle.ordered_scatter(key, x, np.zeros(0))[1] is True


@pytest.mark.parametrize("s", [40, 48])
def test_net_axis_golden(golden, s):
    """Per-net loss and gradient against the reference's loop over the nets."""
    g = golden("net")
    loss, grad = oracle.net_axis(g[f"w_{s}"], g[f"x_{s}"], g[f"y_{s}"], g[f"mask_{s}"])
    close(loss, g[f"loss_{s}"])
    close(grad, g[f"grad_{s}"], rtol=1e-11, atol=1e-12)
    dead = np.repeat(g[f"mask_{s}"] == 0.0, 3, axis=1)
    assert dead.any() and (grad[dead] == 0.0).all()


def test_net_axis_gradient_is_the_loss_slope():
    rng = np.random.default_rng(7)
    w = rng.normal(size=(3, 24)) * 0.7
    x, y = rng.normal(size=(3, 40)), rng.normal(size=(3, 40))
    mask = np.ones((3, 8))
    _loss, grad = oracle.net_axis(w, x, y, mask)
    for net, col in ((0, 0), (1, 7), (2, 23), (1, 14)):
        up, dn = w.copy(), w.copy()
        up[net, col] += 1e-6
        dn[net, col] -= 1e-6
        slope = (oracle.net_axis(up, x, y, mask)[0][net] - oracle.net_axis(dn, x, y, mask)[0][net]) / 2e-6
        assert abs(grad[net, col] - slope) <= 1e-6 * max(1.0, abs(slope))
