"""Seeded synthetic inputs of the five benchmark configurations.

The reference quotes no dataset for these kernels; every input is drawn from
``np.random.default_rng(seed)`` with the shapes and distributions the
benchmark configurations state:

c1 energy      v (3, N) ~ N(0, 1); bar_out = 1; dot_v (3, N) ~ N(0, 1)       N = 2^24
c2 poly_loss   x (N,) ~ U[-2, 2]; t = x + 0.1 N(0, 1); a, b, c = 0.5, -1, 2;
               bar_r = 1; float64 and float32 planes                        N = 2^26
c3 gravity     r1, r2 (3, N) ~ U[-10, 10]^3, pairs closer than 0.1 redrawn;
               m1, m2 ~ U[0.5, 2]; G = 1; dr1, dr2, bar_f (3, N), bar_u ~ N(0, 1)  N = 2^23
c4 spd_solve   A = B B^T + 6 I, B (6, 6) ~ N(0, 1), stored (6, 6, N);
               b, bar_x (6, N) ~ N(0, 1)                                     N = 2^20
c5 kepler      e ~ U[0, 0.95], M ~ U[0, 2 pi); bar_E ~ N(0, 1)               N = 2^24

Planes are component-major with samples last, as the kernels bind them.
"""

from __future__ import annotations

import numpy as np

FULL_N = {"energy": 1 << 24, "poly_loss": 1 << 26, "gravity": 1 << 23, "spd_solve": 1 << 20, "kepler": 1 << 24,
          "oscillator": 1 << 22, "orbit": 1 << 20}


def energy(n: int, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((3, n))
    dot_v = rng.standard_normal((3, n))
    return {"v": v, "bar_out": np.ones(n), "dot_v": dot_v}


def poly_loss(n: int, seed: int = 0, dtype=np.float64) -> dict:
    rng = np.random.default_rng(seed)
    x = rng.uniform(-2.0, 2.0, n)
    t = x + 0.1 * rng.standard_normal(n)
    return {"x": x.astype(dtype), "t": t.astype(dtype), "a": 0.5, "b": -1.0, "c": 2.0,
            "bar_r": np.ones(n, dtype=dtype)}


def gravity(n: int, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    r1 = rng.uniform(-10.0, 10.0, (3, n))
    r2 = rng.uniform(-10.0, 10.0, (3, n))
    while True:
        close = np.sqrt(((r1 - r2) ** 2).sum(axis=0)) < 0.1
        k = int(close.sum())
        if k == 0:
            break
        r1[:, close] = rng.uniform(-10.0, 10.0, (3, k))
        r2[:, close] = rng.uniform(-10.0, 10.0, (3, k))
    return {"r1": r1, "r2": r2, "m1": rng.uniform(0.5, 2.0, n), "m2": rng.uniform(0.5, 2.0, n), "G": 1.0,
            "dr1": rng.standard_normal((3, n)), "dr2": rng.standard_normal((3, n)),
            "bar_f": rng.standard_normal((3, n)), "bar_u": rng.standard_normal(n)}


def spd_solve(n: int, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    B = rng.standard_normal((n, 6, 6))
    A = np.einsum("nij,nkj->nik", B, B) + 6.0 * np.eye(6)
    A = np.ascontiguousarray(np.moveaxis(A, 0, -1))          # (6, 6, N)
    return {"A": A, "b": rng.standard_normal((6, n)), "bar_x": rng.standard_normal((6, n))}


def kepler(n: int, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    return {"e": rng.uniform(0.0, 0.95, n), "M": rng.uniform(0.0, 2.0 * np.pi, n),
            "bar_E": rng.standard_normal(n)}


def trig(n: int, seed: int = 0) -> dict:
    """Arguments of sin/cos: x ~ U[0, 2 pi) (the range Kepler's Newton trips take)."""
    rng = np.random.default_rng(seed)
    return {"x": rng.uniform(0.0, 2.0 * np.pi, n)}


def oscillator(n: int, seed: int = 0, stop_max: int = 64, done_every: int = 0) -> dict:
    """Damped oscillators: w in [0.5, 3], z in [0, 0.3], x(0) ~ N(0, 1), v(0) = 0,
    each stopping after its own 1..stop_max steps; every ``done_every``-th sample
    starts finished (0: none).  dt = 0.01."""
    rng = np.random.default_rng(seed)
    term = np.zeros(n, dtype=bool)
    if done_every:
        term[3::done_every] = True
    return {"omega": rng.uniform(0.5, 3.0, n), "zeta": rng.uniform(0.0, 0.3, n),
            "nstop": rng.integers(1, stop_max + 1, n).astype(np.float64), "x": rng.standard_normal(n),
            "v": np.zeros(n), "k": np.zeros(n), "terminated": term, "dt": 0.01}


def orbit(n: int, seed: int = 0, done_every: int = 0) -> dict:
    """Two-body orbits (GM = 1, semi-major axis 1): eccentricity in [0, 0.7],
    starting at periapsis in a random orientation, integrated from t = 0 to
    t_end in [0.5, 2 pi] with a first step h in [0.02, 0.5] (the larger ones
    are rejected before the controller settles)."""
    rng = np.random.default_rng(seed)
    e = rng.uniform(0.0, 0.7, n)
    rp = 1.0 - e
    vp = np.sqrt((1.0 + e) / (1.0 - e))
    # a random orthonormal frame per sample: periapsis direction p, velocity direction q
    a = rng.standard_normal((3, n))
    p = a / np.linalg.norm(a, axis=0)
    b = rng.standard_normal((3, n))
    b -= p * np.sum(b * p, axis=0)
    q = b / np.linalg.norm(b, axis=0)
    s = np.concatenate([p * rp, q * vp])
    term = np.zeros(n, dtype=bool)
    if done_every:
        term[3::done_every] = True
    return {"s": np.ascontiguousarray(s), "t": np.zeros(n), "h": rng.uniform(0.02, 0.5, n), "n_acc": np.zeros(n),
            "n_rej": np.zeros(n), "t_end": rng.uniform(0.5, 2.0 * np.pi, n), "terminated": term}


#: Samples per segment of the segment_sum kernel (its key is sample // SEGMENT).
SEGMENT = 256


def scatter(n: int, seed: int = 0, slots: int = 1000) -> dict:
    """Terms x ~ U[0.5, 1.5] (positive: the per-slot bound is relative to the
    sum), keys uniform over ``slots`` (``key``), the same keys sorted
    (``sorted_key``), a table of ``slots`` values with indices that also fall
    outside it (clamped), and 32-bit words with one random bit each."""
    rng = np.random.default_rng(seed)
    key = rng.integers(0, slots, n).astype(np.int32)
    return {"x": rng.uniform(0.5, 1.5, n), "key": key, "sorted_key": np.sort(key),
            "idx": rng.integers(-3, slots + 3, n).astype(np.int32), "w": rng.standard_normal(n),
            "table": rng.standard_normal(slots), "bar_y": rng.uniform(0.5, 1.5, n),
            "bits": (np.uint32(1) << rng.integers(0, 32, n).astype(np.uint32)).astype(np.uint32), "slots": slots}


#: The lane given an input its factorisation fails on, in the team workloads.
TEAM_BAD = 2


def team(n: int, lanes: int, kind: str, seed: int = 0, bad: int | None = TEAM_BAD) -> dict:
    """Per-lane n x n matrices (A, (n, n, lanes)), a right-hand side b (n, lanes)
    and a two-column one B (n, 2, lanes), the distributions of the reference's
    team-form tests: ``spd`` g g^T + I with g ~ N(0, 1/n) (lane ``bad``: a
    negative diagonal entry at n // 2, so the leading minor n // 2 + 1 fails);
    ``general`` N(0, 1/n) + 0.5 I (lane ``bad``: column 1 zero, singular);
    ``lower`` a lower triangle with diagonal in [1, 2) and noise above it, which
    chol_from ignores (lane ``bad``: a zero first diagonal entry)."""
    rng = np.random.default_rng(seed)
    mats = np.empty((lanes, n, n))
    for lane in range(lanes):
        if kind == "spd":
            g = rng.standard_normal((n, n)) / np.sqrt(n)
            a = g @ g.T + np.eye(n)
            if lane == bad:
                a[n // 2, n // 2] = -1.0
        elif kind == "general":
            a = rng.standard_normal((n, n)) / np.sqrt(n) + 0.5 * np.eye(n)
            if lane == bad:
                a[:, min(1, n - 1)] = 0.0
        elif kind == "lower":
            a = np.tril(rng.standard_normal((n, n)), -1) / np.sqrt(n) + np.diag(1.0 + rng.random(n))
            a += 0.5 * np.triu(rng.standard_normal((n, n)), 1)
            if lane == bad:
                a[0, 0] = 0.0
        else:
            raise ValueError(kind)
        mats[lane] = a
    return {"A": np.ascontiguousarray(np.moveaxis(mats, 0, -1)),
            "b": np.ascontiguousarray(rng.standard_normal((n, lanes))),
            "B": np.ascontiguousarray(rng.standard_normal((n, 2, lanes)))}


MAKERS = {"energy": energy, "poly_loss": poly_loss, "gravity": gravity, "spd_solve": spd_solve, "kepler": kepler,
          "trig": trig, "oscillator": oscillator, "orbit": orbit, "scatter": scatter}
