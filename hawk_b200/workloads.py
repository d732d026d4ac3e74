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

FULL_N = {"energy": 1 << 24, "poly_loss": 1 << 26, "gravity": 1 << 23, "spd_solve": 1 << 20, "kepler": 1 << 24}


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


MAKERS = {"energy": energy, "poly_loss": poly_loss, "gravity": gravity, "spd_solve": spd_solve, "kepler": kepler}
