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
   band_rows       s = hawk.sum(x), q = hawk.sum(x * x), in the banded scalar mode
   band_max/min    hi = hawk.max(x) / lo = hawk.min(x), banded
   band_chain      out = exp(x x / 2 + y) / (y + 1.5) - sin(x) / 4, banded and float64
   trig            s = sin(x), c = cos(x): the device library's sin and cos
                   as output planes, for the bitwise check against the host
                   target's libm

Stepping kernels (automatic, ``steps="auto"``: each launch runs up to the
``fused_steps`` word of steps per sample, a sample leaving at its own finish;
hawk/trace/steps.py):

s1 oscillator      one classic RK4 step of x'' = -w^2 x - 2 z w x' per step,
                   finishing at the sample's own stop step
s2 orbit           one adaptive Fehlberg 7(8) attempt on the two-body problem
                   (GM = 1) per step, finishing at the sample's final time;
                   the step-size factor is 0.9 * err^(-1/8), clamped to
                   [0.2, 5], with err^(-1/8) taken as three square roots

Scattered commits (hawk.scatter, the VJP of a table read; several samples add
into one slot, hk/accum.cuh):

g1 gather          y = w * table[idx]; its VJP adds bar_y * w into bar_table[idx]
g2 segment_sum     acc[i / 256] += x, the default (compensated) policy: the key
                   is constant over aligned runs of lanes
g3 keyed_sum       acc[key] += x over a Sorted key (runs found per warp)
g4 histogram       acc[key] += x over any key, compensated
g5 bitmask         acc[key] |= bits (32-bit words)
g6 comp_scatter    acc[key] += x under the compensated sink policy (a Kind):
                   each add's rounding error committed into the kernel's own
                   companion plane acc_c
"""

from __future__ import annotations

from .frontend import load

hawk = load()

import hawk.math as m  # noqa: E402
from hawk import Grid, Index, Int32, Kernel, Matrix, Mutable, Param, Scalar, Sorted, Table, Terminated, UInt32, Vector  # noqa: E402,E501
from hawk.diff import jvp, param_planes, vjp  # noqa: E402
from hawk.ext import Kind, sink_policy  # noqa: E402


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


@hawk.kernel
def band_rows(x: Scalar, s: Mutable[Scalar], q: Mutable[Scalar]):
    s = hawk.sum(x)
    q = hawk.sum(x * x)


@hawk.kernel
def band_max(x: Scalar, hi: Mutable[Scalar]):
    hi = hawk.max(x)


@hawk.kernel
def band_min(x: Scalar, lo: Mutable[Scalar]):
    lo = hawk.min(x)


@hawk.kernel
def band_chain(x: Scalar, y: Scalar, out: Mutable[Scalar]):
    t = x * x * 0.5 + y
    out = m.exp(t) / (y + 1.5) - m.sin(x) * 0.25


@hawk.kernel
def trig(x: Scalar, s: Mutable[Scalar], c: Mutable[Scalar]):
    s = m.sin(x)
    c = m.cos(x)


def _rk4_accel(stiff, damp, p, q):
    return stiff * p - damp * q


@hawk.kernel
def oscillator(omega: Scalar, zeta: Scalar, nstop: Scalar, dt: Param, terminated: Terminated,
               x: Mutable[Scalar], v: Mutable[Scalar], k: Mutable[Scalar]):
    x0 = x
    v0 = v
    stiff = -(omega * omega)
    damp = 2.0 * zeta * omega
    half = 0.5 * dt
    a1 = _rk4_accel(stiff, damp, x0, v0)
    v2 = v0 + half * a1
    a2 = _rk4_accel(stiff, damp, x0 + half * v0, v2)
    v3 = v0 + half * a2
    a3 = _rk4_accel(stiff, damp, x0 + half * v2, v3)
    v4 = v0 + dt * a3
    a4 = _rk4_accel(stiff, damp, x0 + dt * v3, v4)
    sixth = dt / 6.0
    x = x0 + sixth * (v0 + 2.0 * (v2 + v3) + v4)
    v = v0 + sixth * (a1 + 2.0 * (a2 + a3) + a4)
    kn = k + 1.0
    k = kn
    terminated = kn >= nstop


#: Fehlberg's 7(8) pair (NASA TR R-287, 1968): the stage matrix (row j: the
#: weights of stages 0 .. j-1 in stage j), the 8th-order weights, and the
#: error weight 41/840 of stages 0, 10, 11, 12 (+, +, -, -).
RKF78_A = (
    (2.0 / 27.0,),
    (1.0 / 36.0, 1.0 / 12.0),
    (1.0 / 24.0, 0.0, 1.0 / 8.0),
    (5.0 / 12.0, 0.0, -25.0 / 16.0, 25.0 / 16.0),
    (1.0 / 20.0, 0.0, 0.0, 1.0 / 4.0, 1.0 / 5.0),
    (-25.0 / 108.0, 0.0, 0.0, 125.0 / 108.0, -65.0 / 27.0, 125.0 / 54.0),
    (31.0 / 300.0, 0.0, 0.0, 0.0, 61.0 / 225.0, -2.0 / 9.0, 13.0 / 900.0),
    (2.0, 0.0, 0.0, -53.0 / 6.0, 704.0 / 45.0, -107.0 / 9.0, 67.0 / 90.0, 3.0),
    (-91.0 / 108.0, 0.0, 0.0, 23.0 / 108.0, -976.0 / 135.0, 311.0 / 54.0, -19.0 / 60.0, 17.0 / 6.0,
     -1.0 / 12.0),
    (2383.0 / 4100.0, 0.0, 0.0, -341.0 / 164.0, 4496.0 / 1025.0, -301.0 / 82.0, 2133.0 / 4100.0,
     45.0 / 82.0, 45.0 / 164.0, 18.0 / 41.0),
    (3.0 / 205.0, 0.0, 0.0, 0.0, 0.0, -6.0 / 41.0, -3.0 / 205.0, -3.0 / 41.0, 3.0 / 41.0, 6.0 / 41.0, 0.0),
    (-1777.0 / 4100.0, 0.0, 0.0, -341.0 / 164.0, 4496.0 / 1025.0, -289.0 / 82.0, 2193.0 / 4100.0,
     51.0 / 82.0, 33.0 / 164.0, 12.0 / 41.0, 0.0, 1.0),
)
RKF78_B = {5: 34.0 / 105.0, 6: 9.0 / 35.0, 7: 9.0 / 35.0, 8: 9.0 / 280.0, 9: 9.0 / 280.0,
           11: 41.0 / 840.0, 12: 41.0 / 840.0}
RKF78_ERR = ((0, 1.0), (10, 1.0), (11, -1.0), (12, -1.0))
ORBIT_TOL = 1e-10


def _orbit_rate(s):
    """d/dt of the two-body state (position, velocity) with GM = 1."""
    rr = s[0] * s[0] + s[1] * s[1] + s[2] * s[2]
    w = 1.0 / (rr * m.sqrt(rr))
    return [s[3], s[4], s[5], -(s[0] * w), -(s[1] * w), -(s[2] * w)]


def _weighted(terms):
    """sum of weight * stage over the nonzero weights, in stage order."""
    acc = None
    for wgt, val in terms:
        t = wgt * val
        acc = t if acc is None else acc + t
    return acc


def _rkf78(s0, h):
    """The 8th-order state and the error estimate of one attempt of step h."""
    ks = [_orbit_rate(s0)]
    for row in RKF78_A:
        y = [s0[d] + h * _weighted([(a, ks[j][d]) for j, a in enumerate(row) if a != 0.0])
             for d in range(6)]
        ks.append(_orbit_rate(y))
    s8 = [s0[d] + h * _weighted([(b, ks[j][d]) for j, b in sorted(RKF78_B.items())]) for d in range(6)]
    err = [h * (41.0 / 840.0) * _weighted([(sg, ks[j][d]) for j, sg in RKF78_ERR]) for d in range(6)]
    return s8, err


def _err_norm(s0, s8, err):
    """max over components of |err| / (tol + tol * max(|s8|, |s0|))."""
    worst = None
    for d in range(6):
        q = m.abs(err[d]) / (ORBIT_TOL + ORBIT_TOL * m.max(m.abs(s8[d]), m.abs(s0[d])))
        worst = q if worst is None else m.max(worst, q)
    return worst


@hawk.kernel
def orbit(t_end: Scalar, terminated: Terminated, s: Mutable[Vector[6]], t: Mutable[Scalar],
          h: Mutable[Scalar], n_acc: Mutable[Scalar], n_rej: Mutable[Scalar]):
    s0 = s
    t0 = t
    rest = t_end - t0
    final = h >= rest
    step = m.where(final, rest, h)
    s8, err = _rkf78(s0, step)
    worst = _err_norm(s0, s8, err)
    ok = worst < 1.0
    shrink = 1.0 / m.sqrt(m.sqrt(m.sqrt(worst)))
    h = step * m.min(5.0, m.max(0.2, 0.9 * shrink))
    s = m.where(ok, m.vec(s8), s0)
    t_next = m.where(ok, m.where(final, t_end, t0 + step), t0)
    t = t_next
    n_acc = n_acc + m.where(ok, 1.0, 0.0)
    n_rej = n_rej + m.where(ok, 0.0, 1.0)
    terminated = t_next >= t_end


from .workloads import SEGMENT  # noqa: E402  -- samples per segment of segment_sum


@hawk.kernel
def gather(idx: Index, w: Scalar, table: Table[Scalar], y: Mutable[Scalar]):
    y = w * table[idx]


@hawk.kernel
def segment_sum(x: Scalar, acc: Mutable[Scalar]):
    seg, _pos = m.split_index(SEGMENT)
    hawk.scatter(acc)[seg] += x


@hawk.kernel
def keyed_sum(x: Scalar, key: Sorted[Index], acc: Mutable[Scalar]):
    hawk.scatter(acc, policy="plain")[key] += x


@hawk.kernel
def histogram(x: Scalar, key: Index, acc: Mutable[Scalar]):
    hawk.scatter(acc, policy="compensated")[key] += x


@hawk.kernel
def bitmask(bits: UInt32, key: Index, acc: Mutable[UInt32]):
    hawk.scatter(acc, policy="or")[key] |= bits


#: The compensated sink policy (hawk/ext): the scatter's plain commit into acc
#: becomes a compensated one whose residuals go to the declared plane acc_c.
COMPENSATED_SINK = Kind("compensated", sink=sink_policy("compensated", into="acc_c"))


@hawk.kernel(kind=COMPENSATED_SINK)
def comp_scatter(x: Scalar, key: Index, acc: Mutable[Scalar], acc_c: Mutable[Scalar]):
    hawk.scatter(acc, policy="plain")[key] += x
    hawk.scatter(acc_c, policy="plain")[key] += 0.0


@hawk.kernel
def team_chol_33(A: Matrix[33, 33], b: Vector[33], B: Matrix[33, 2], x: Mutable[Vector[33]],
                 X: Mutable[Matrix[33, 2]], L: Mutable[Matrix[33, 33]], info: Mutable[Int32]):
    f, status = m.cholesky(A)
    x = m.cho_solve(f, b)
    X = m.cho_solve(f, B)
    L = f
    info = status


@hawk.kernel
def team_lu_33(A: Matrix[33, 33], b: Vector[33], B: Matrix[33, 2], x: Mutable[Vector[33]],
               X: Mutable[Matrix[33, 2]], det: Mutable[Scalar], info: Mutable[Int32]):
    f, status = m.lu(A)
    x = m.lu_solve(f, b)
    X = m.lu_solve(f, B)
    det = m.det(A)
    info = status


@hawk.kernel
def team_chol_64(A: Matrix[64, 64], b: Vector[64], B: Matrix[64, 2], x: Mutable[Vector[64]],
                 X: Mutable[Matrix[64, 2]], L: Mutable[Matrix[64, 64]], info: Mutable[Int32]):
    f, status = m.cholesky(A)
    x = m.cho_solve(f, b)
    X = m.cho_solve(f, B)
    L = f
    info = status


@hawk.kernel
def team_lu_64(A: Matrix[64, 64], b: Vector[64], B: Matrix[64, 2], x: Mutable[Vector[64]],
               X: Mutable[Matrix[64, 2]], det: Mutable[Scalar], info: Mutable[Int32]):
    f, status = m.lu(A)
    x = m.lu_solve(f, b)
    X = m.lu_solve(f, B)
    det = m.det(A)
    info = status


@hawk.kernel
def team_chol_128(A: Matrix[128, 128], b: Vector[128], B: Matrix[128, 2], x: Mutable[Vector[128]],
                  X: Mutable[Matrix[128, 2]], L: Mutable[Matrix[128, 128]], info: Mutable[Int32]):
    f, status = m.cholesky(A)
    x = m.cho_solve(f, b)
    X = m.cho_solve(f, B)
    L = f
    info = status


@hawk.kernel
def team_lu_128(A: Matrix[128, 128], b: Vector[128], B: Matrix[128, 2], x: Mutable[Vector[128]],
                X: Mutable[Matrix[128, 2]], det: Mutable[Scalar], info: Mutable[Int32]):
    f, status = m.lu(A)
    x = m.lu_solve(f, b)
    X = m.lu_solve(f, B)
    det = m.det(A)
    info = status


@hawk.kernel
def team_chol_from_64(A: Matrix[64, 64], b: Vector[64], x: Mutable[Vector[64]], L: Mutable[Matrix[64, 64]],
                      info: Mutable[Int32]):
    f, status = m.chol_from(A)
    x = m.cho_solve(f, b)
    L = f
    info = status


@hawk.kernel
def share(x: Scalar, z: Mutable[Scalar]):
    z = x / hawk.sum(x)


@hawk.kernel
def standard(x: Scalar, mu: Mutable[Scalar], z: Mutable[Scalar], t: Mutable[Scalar]):
    mu = hawk.mean(x)
    v = hawk.mean((x - mu) * (x - mu))
    z = (x - mu) / m.sqrt(v)
    t = hawk.sum(z * z)


@hawk.kernel
def centred(x: Scalar, z: Mutable[Vector[3]]):
    v = m.vec(x, x * x, 2.0 * x)
    z = v - hawk.mean(v)


@hawk.kernel
def key_total(lane: Grid["key", "row":8], x: Scalar) -> Scalar:
    return hawk.sum(x, over="row")


@hawk.kernel
def key_share(lane: Grid["key", "row":8], x: Scalar, z: Mutable[Scalar]):
    z = x / hawk.sum(x, over="row")


@hawk.kernel
def gram_block(lane: Grid["key", "row":8], j: Vector[6]) -> Matrix[6, 6]:
    return hawk.sum(m.outer(j, j), over="row")


@hawk.kernel
def grad_block(lane: Grid["key", "row":8], j: Vector[20], r: Scalar) -> Vector[20]:
    return hawk.sum(j * r, over="row")


@hawk.kernel
def ordered_total(lane: Grid["key", "row":8], x: Scalar) -> Scalar:
    return hawk.sum(x, over="row", policy="ordered")


@hawk.kernel
def ordered_long(lane: Grid["key", "row":197385], x: Scalar) -> Scalar:
    return hawk.sum(x, over="row", policy="ordered")


@hawk.kernel
def ordered_hist(x: Scalar, key: Index, acc: Mutable[Scalar]):
    hawk.scatter(acc, policy="ordered")[key] += x


#: The named net axis: K small models in one launch (the reference's
#: tests/_net_axis_kernels.py:16-27).  Lanes are (net, sample); W[net, :]
#: holds each net's (a, b, c) per hidden unit, a mask row zeroes the unused
#: units of a narrower net; the loss keeps the net label.  Its gradient wrt W
#: is a keyed accumulate into the table: atomic per-warp partials by default,
#: and under policy="ordered" a per-lane log folded per key in lane order by a
#: team stage (hawk/diff/ordered.py, hawk/ir/team.py:677-693).
NET_HIDDEN, NET_WEIGHTS = 8, 24


def net_loss_for(samples: int, policy: str = "compensated") -> Kernel:
    @hawk.kernel
    def net_loss(lane: Grid["net", "sample":samples], W: Table["net", "p":NET_WEIGHTS],
                 mask: Table["net", "h":NET_HIDDEN], x: Scalar, y: Scalar) -> Scalar:
        pred = 0.0 * x
        for h in range(NET_HIDDEN):
            a = W.at(net=lane.net, p=3 * h)
            b = W.at(net=lane.net, p=3 * h + 1)
            c = W.at(net=lane.net, p=3 * h + 2)
            pred = pred + mask.at(net=lane.net, h=h) * c * m.tanh(a * x + b)
        return hawk.sum((pred - y) * (pred - y), over="sample", policy=policy)

    return Kernel(f"net_loss_{samples}" + ("_ordered" if policy == "ordered" else ""),
                  net_loss.sinks, net_loss.planes)


NET_KERNELS = {}
for _s, _policy in ((40, "compensated"), (40, "ordered"), (48, "ordered")):
    _loss = net_loss_for(_s, _policy)
    _grad_name = _loss.name.replace("net_loss", "net_grad")
    NET_KERNELS[_loss.name] = _loss
    NET_KERNELS[_grad_name] = Kernel(_grad_name, vjp(_loss, wrt=("W",)))


#: Sums over some lane axes (hawk.sum(x, over=...), hawk/trace/reduce.py:
#: one value per kept key): returned as an output, or read back in the body at
#: the lane's own key (a keyed plane the runtime owns between two stages); a
#: per-key block of more than 16 entries (an outer product's Gram block, a
#: gradient of 20) is a BlockSum: the rows stored by a per-lane stage, each
#: key's block summed in lane order by a team stage (hawk/ir/team.py:544-600).
#: Under policy="ordered" a plain per-key sum, and a scatter by any key, are
#: folded without atomics in fixed orders by the reference's ordered stages
#: (hawk/ir/team.py:602-720): the same bits on every launch.
KEYED_KERNELS = {k.name: k for k in (key_total, key_share, gram_block, grad_block, ordered_total, ordered_long,
                                          ordered_hist)}


#: Sums over samples read back in the body (hawk/ir/split.py): each runs as
#: stages with the cell finished on the device between them -- x / sum(x),
#: the standardised x with its mean stored and the sum of squares of the
#: result, a vector's components centred on their means.
READBACK_KERNELS = {k.name: k for k in (share, standard, centred)}


@hawk.kernel
def sym_eigen(A: Matrix[6, 6], w: Mutable[Vector[6]], V: Mutable[Matrix[6, 6]], info: Mutable[Int32]):
    vals, vecs, status = m.eigh(A)
    w = vals
    V = vecs
    info = status


@hawk.kernel
def sym_eigvals(A: Matrix[4, 4], w: Mutable[Vector[4]], info: Mutable[Int32]):
    vals, _vecs, status = m.eigh(A)
    w = vals
    info = status


@hawk.kernel
def team_eigh_40(A: Matrix[40, 40], w: Mutable[Vector[40]], V: Mutable[Matrix[40, 40]], info: Mutable[Int32]):
    vals, vecs, status = m.eigh(A)
    w = vals
    V = vecs
    info = status


@hawk.kernel
def team_lstsq_40(J: Matrix[80, 40], r: Vector[80], x: Mutable[Vector[40]], info: Mutable[Int32]):
    sol, status = m.lstsq(J, r)
    x = sol
    info = status


@hawk.kernel
def team_chol_512(A: Matrix[512, 512], b: Vector[512], x: Mutable[Vector[512]], info: Mutable[Int32]):
    f, status = m.cholesky(A)
    x = m.cho_solve(f, b)
    info = status


@hawk.kernel
def team_lu_160(A: Matrix[160, 160], b: Vector[160], x: Mutable[Vector[160]], det: Mutable[Scalar],
                info: Mutable[Int32]):
    f, status = m.lu(A)
    x = m.lu_solve(f, b)
    det = m.det(A)
    info = status


@hawk.kernel
def warp_eigvals_32(A: Matrix[32, 32], w: Mutable[Vector[32]], info: Mutable[Int32]):
    vals, _vecs, status = m.eigh(A)
    w = vals
    info = status


#: The team-form kernels: per sample, Cholesky solves (x, X, the factor L and
#: its status) and LU solves with partial pivoting (x, X, det(A) -- its own
#: factor, as hawk.math.det spells it -- and the status), at sizes above the
#: one-thread cap of 32 (hawk/ir/linalg.py:33-36), and solves against a given
#: lower-triangular factor (chol_from).  At 512 (Cholesky) and 160 (LU) the
#: matrix does not fit a block's shared memory and the team works it in place
#: in its scratch plane.
TEAM_KERNELS = {k.name: k for k in (team_chol_33, team_lu_33, team_chol_64, team_lu_64, team_chol_128,
                                    team_lu_128, team_chol_from_64, team_chol_512, team_lu_160, team_eigh_40,
                                    team_lstsq_40, warp_eigvals_32)}


#: Every kernel the bundles hold, by name, with the scalar modes each is built in.
KERNELS = {
    "energy": (energy, ("float64",)),
    "energy_vjp": (Kernel("energy_vjp", vjp(energy, wrt=("v",))), ("float64",)),
    "energy_jvp": (Kernel("energy_jvp", jvp(energy, wrt=("v",))), ("float64",)),
    "poly_loss": (poly_loss, ("float64", "float32")),
    "poly_loss_vjp": (Kernel("poly_loss_vjp", vjp(param_planes(poly_loss), wrt=("a", "b", "c"))),
                      ("float64", "float32", "banded")),
    "gravity": (gravity, ("float64",)),
    "gravity_jvp": (Kernel("gravity_jvp", jvp(gravity, wrt=("r1", "r2"))), ("float64",)),
    "gravity_vjp": (Kernel("gravity_vjp", vjp(gravity, wrt=("r1", "r2"))), ("float64",)),
    "spd_solve": (spd_solve, ("float64",)),
    "spd_solve_vjp": (Kernel("spd_solve_vjp", vjp(spd_solve, wrt=("A", "b"))), ("float64",)),
    "kepler": (kepler, ("float64",)),
    "kepler_vjp": (Kernel("kepler_vjp", vjp(kepler, wrt=("e", "M"))), ("float64",)),
    "trig": (trig, ("float64",)),
    "band_rows": (band_rows, ("banded", "float64")),
    "band_max": (band_max, ("banded",)),
    "band_min": (band_min, ("banded",)),
    "band_chain": (band_chain, ("banded", "float64")),
    "oscillator": (oscillator, ("float64",)),
    "orbit": (orbit, ("float64",)),
    "gather": (gather, ("float64",)),
    "gather_vjp": (Kernel("gather_vjp", vjp(gather, wrt=("table", "w"))), ("float64",)),
    "segment_sum": (segment_sum, ("float64",)),
    "keyed_sum": (keyed_sum, ("float64",)),
    "histogram": (histogram, ("float64",)),
    "bitmask": (bitmask, ("float64",)),
    "comp_scatter": (comp_scatter, ("float64",)),
    **{name: (k, ("float64", "float32") if name == "warp_eigvals_32" else ("float64",))
       for name, k in TEAM_KERNELS.items()},
    **{name: (k, ("float64",)) for name, k in READBACK_KERNELS.items()},
    **{name: (k, ("float64",)) for name, k in KEYED_KERNELS.items()},
    **{name: (k, ("float64",)) for name, k in NET_KERNELS.items()},
    "share_vjp": (Kernel("share_vjp", vjp(share, wrt=("x",))), ("float64",)),
    "sym_eigen": (sym_eigen, ("float64",)),
    "sym_eigvals": (sym_eigvals, ("float64",)),
}
