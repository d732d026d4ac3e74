"""The five benchmark kernels, written as hawk user code.

Each is a plain ``@hawk.kernel`` for one sample, with its derivatives taken by
the reference's own ``hawk.diff.vjp`` / ``jvp`` / ``param_planes``
(hawk/diff/transform.py:241, :469; hawk/diff/params.py:57).  Importing this
module brings up the reference's front end (``hawk_b200.frontend``); the
runtime never imports it -- it loads the bundles built from these kernels.

c1 energy          out = 0.5 * dot(v, v)                       (README.md:80-99)
c2 poly_loss       r = (a*x^3 + b*x + c - t)^2, Params a, b, c; VJP wrt the
                   Params promoted to one-cell planes, so each gradient is a
                   sum over samples (32-sample rows + the ordered finish)
c3 gravity         f = G m1 m2 / |d|^3 * d, u = -G m1 m2 / |d|, d = r2 - r1
c4 spd_solve       x = cho_solve(cholesky(A), b) for a 6x6 SPD A
c5 kepler          Newton on E - e sin E = M from E = M, at most 32 trips,
                   leaving when |dE| < 1e-14; E and the trip count (int32)
"""

from __future__ import annotations

from .frontend import load

hawk = load()

import hawk.math as m  # noqa: E402
from hawk import Int32, Kernel, Matrix, Mutable, Param, Scalar, Vector  # noqa: E402
from hawk.diff import jvp, param_planes, vjp  # noqa: E402


@hawk.kernel
def energy(v: Vector[3], out: Mutable[Scalar]):
    out = 0.5 * m.dot(v, v)


@hawk.kernel
def poly_loss(x: Scalar, t: Scalar, a: Param, b: Param, c: Param, r: Mutable[Scalar]):
    y = a * x * x * x + b * x + c
    d = y - t
    r = d * d


@hawk.kernel
def gravity(r1: Vector[3], r2: Vector[3], m1: Scalar, m2: Scalar, G: Param,
            f: Mutable[Vector[3]], u: Mutable[Scalar]):
    d = r2 - r1
    dist = m.norm(d)
    gm = G * m1 * m2
    f = (gm / (dist * dist * dist)) * d
    u = -gm / dist


@hawk.kernel
def spd_solve(A: Matrix[6, 6], b: Vector[6], x: Mutable[Vector[6]]):
    L, _info = m.cholesky(A)
    x = m.cho_solve(L, b)


@hawk.kernel
def kepler(e: Scalar, M: Scalar, E: Mutable[Scalar], iters: Mutable[Int32]):
    Ek = M
    n = m.int32(0)
    for _k in range(32):
        dE = (Ek - e * m.sin(Ek) - M) / (1.0 - e * m.cos(Ek))
        Ek = Ek - dE
        n = n + 1
        if m.abs(dE) < 1e-14:
            break
    E = Ek
    iters = n


#: Every kernel the bundles hold, by name, with the scalar modes each is built in.
KERNELS = {
    "energy": (energy, ("float64",)),
    "energy_vjp": (Kernel("energy_vjp", vjp(energy, wrt=("v",))), ("float64",)),
    "energy_jvp": (Kernel("energy_jvp", jvp(energy, wrt=("v",))), ("float64",)),
    "poly_loss": (poly_loss, ("float64", "float32")),
    "poly_loss_vjp": (Kernel("poly_loss_vjp", vjp(param_planes(poly_loss), wrt=("a", "b", "c"))),
                      ("float64", "float32")),
    "gravity": (gravity, ("float64",)),
    "gravity_jvp": (Kernel("gravity_jvp", jvp(gravity, wrt=("r1", "r2"))), ("float64",)),
    "gravity_vjp": (Kernel("gravity_vjp", vjp(gravity, wrt=("r1", "r2"))), ("float64",)),
    "spd_solve": (spd_solve, ("float64",)),
    "spd_solve_vjp": (Kernel("spd_solve_vjp", vjp(spd_solve, wrt=("A", "b"))), ("float64",)),
    "kepler": (kepler, ("float64",)),
    "kepler_vjp": (Kernel("kepler_vjp", vjp(kepler, wrt=("e", "M"))), ("float64",)),
}
