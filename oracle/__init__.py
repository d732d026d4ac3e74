"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the b200 path.

A plain-C restatement (hawk_oracle.c) of what the reference's host target
computes for the five benchmark kernels, loaded with ctypes.  Only the tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
package -- as the checker and the timed CPU baseline, never as part of the
product path.

Parity is pinned by golden vectors made from the reference's own numpy IR
interpreter (tests/_eval.py in the reference, run on the reference's traced and
derived IR; tests/golden/make_golden.py) and by the reference's known answers
(README.md:80-99 energy; the Kepler (e=0.5, M=1) root).

The library is built per host CPU (``-march=native`` like the reference's
`native` host profile), on first use, under ``oracle/_build/<cpu key>/``.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OP = {"sum": 0, "max": 1, "min": 2}
_LOCK = threading.Lock()
_LIB = None


def _cpu_key() -> str:
    try:
        text = Path("/proc/cpuinfo").read_text()
    except OSError:
        text = ""
    model = next((ln.split(":", 1)[1].strip() for ln in text.splitlines() if ln.startswith("model name")), "")
    flags = next((ln.split(":", 1)[1].strip() for ln in text.splitlines() if ln.startswith("flags")), "")
    return hashlib.sha256((model + "|" + flags).encode()).hexdigest()[:12]


def library_path() -> Path:
    return HERE / "_build" / _cpu_key() / "libhawk_oracle.so"


def build() -> Path:
    """Compile the oracle for this host's CPU (once)."""
    out = library_path()
    src = [HERE / "hawk_oracle.c", HERE / "hawk_oracle.h"]
    if out.exists() and out.stat().st_mtime >= max(p.stat().st_mtime for p in src):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O3", "-march=native", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-std=c11",
           "-shared", str(HERE / "hawk_oracle.c"), "-o", str(out), "-lm"]
    env = dict(os.environ)
    env.pop("CC", None)
    run = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if run.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{run.stderr}")
    return out


_P = ctypes.c_void_p
_I = ctypes.c_int64
_D = ctypes.c_double
_F = ctypes.c_float
_SIGS = {
    "hko_energy": (None, [_P, _I, _P, _I, _I]),
    "hko_energy_vjp": (None, [_P, _I, _P, _P, _I, _I, _I]),
    "hko_energy_jvp": (None, [_P, _I, _P, _I, _P, _I, _I]),
    "hko_poly_loss_f64": (None, [_P, _P, _D, _D, _D, _P, _I, _I]),
    "hko_poly_loss_f32": (None, [_P, _P, _F, _F, _F, _P, _I, _I]),
    "hko_poly_loss_vjp_rows_f64": (None, [_P, _P, _P, _D, _D, _D, _I, _I, _I, _P, _P]),
    "hko_poly_loss_vjp_rows_f32": (None, [_P, _P, _P, _F, _F, _F, _I, _I, _I, _P, _P]),
    "hko_cells_finish_f64": (_D, [ctypes.c_int, _P, _P, _I]),
    "hko_cells_finish_f32": (_F, [ctypes.c_int, _P, _P, _I]),
    "hko_cells_leaves_d": (None, [ctypes.c_int, _P, _P, _I, _P, _P]),
    "hko_cells_tree_d": (_D, [ctypes.c_int, _P, _P, _I]),
    "hko_cells_leaves_f": (None, [ctypes.c_int, _P, _P, _I, _P, _P]),
    "hko_cells_tree_f": (_F, [ctypes.c_int, _P, _P, _I]),
    "hko_gravity": (None, [_P, _P, _I, _P, _P, _D, _P, _I, _P, _I, _I]),
    "hko_gravity_jvp": (None, [_P, _P, _P, _P, _I, _P, _P, _D, _P, _I, _P, _I, _I]),
    "hko_gravity_vjp": (None, [_P, _P, _P, _I, _P, _P, _P, _D, _P, _P, _I, _I, _I]),
    "hko_spd_solve": (None, [_P, _P, _I, _P, _I, _I, _I]),
    "hko_spd_solve_vjp": (None, [_P, _P, _P, _I, _P, _P, _I, _I, _I]),
    "hko_kepler": (None, [_P, _P, _P, _P, _I, _I]),
    "hko_trig": (None, [_P, _P, _P, _I, _I]),
    "hko_kepler_vjp": (None, [_P, _P, _P, _P, _P, _I, _I]),
    "hko_oscillator": (ctypes.c_uint32, [_P, _P, _P, _P, _P, _P, _P, _D, _I, _I, _I]),
    "hko_orbit": (ctypes.c_uint32, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I]),
    "hko_rows_f64": (None, [ctypes.c_int, _P, _I, _P, _P]),
    "hko_lstsq_qr": (None, [ctypes.c_int, ctypes.c_int, _P, _P, _I, _P, _P, _I, _I]),
    "hko_sym_eigen": (None, [ctypes.c_int, _P, _I, _P, _P, _P, _I, _I]),
    "hko_team_chol": (None, [ctypes.c_int, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I]),
    "hko_team_lu": (None, [ctypes.c_int, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I]),
    "hko_team_chol_from": (None, [ctypes.c_int, _P, _P, _I, _P, _P, _P, _I, _I]),
}


def lib() -> ctypes.CDLL:
    global _LIB
    with _LOCK:
        if _LIB is None:
            handle = ctypes.CDLL(str(build()))
            for name, (res, args) in _SIGS.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = handle
        return _LIB


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


def tiles(n: int, threads: int, align: int = 1):
    """Contiguous [base, base+count) tiles of n samples, ``align``-aligned starts
    (eagle's host team tiles the partition the same way, hawk/emit/host.py:8-12)."""
    threads = max(1, int(threads))
    step = -(-n // threads)
    step = -(-step // align) * align
    return [(b, min(step, n - b)) for b in range(0, n, step)] or [(0, 0)]


def parallel(fn, n: int, threads: int = 1, align: int = 1) -> None:
    """Run ``fn(base, count)`` over tiles on ``threads`` host threads (ctypes
    releases the GIL for the duration of each C call)."""
    parts = tiles(n, threads, align)
    if len(parts) == 1:
        fn(*parts[0])
        return
    with ThreadPoolExecutor(len(parts)) as pool:
        list(pool.map(lambda bc: fn(*bc), parts))


# ------------------------------------------------------------- kernels
def energy(v: np.ndarray, threads: int = 1) -> np.ndarray:
    n = v.shape[-1]
    out = np.empty(n)
    parallel(lambda b, c: lib().hko_energy(_p(v), n, _p(out), b, c), n, threads)
    return out


def energy_vjp(v: np.ndarray, bar_out: np.ndarray, threads: int = 1) -> np.ndarray:
    n = v.shape[-1]
    bar_v = np.empty_like(v)
    parallel(lambda b, c: lib().hko_energy_vjp(_p(v), n, _p(bar_out), _p(bar_v), n, b, c), n, threads)
    return bar_v


def energy_jvp(v: np.ndarray, dot_v: np.ndarray, threads: int = 1) -> np.ndarray:
    n = v.shape[-1]
    out = np.empty(n)
    parallel(lambda b, c: lib().hko_energy_jvp(_p(v), n, _p(dot_v), n, _p(out), b, c), n, threads)
    return out


def poly_loss(x, t, a, b, c, threads: int = 1) -> np.ndarray:
    n = x.shape[0]
    r = np.empty_like(x)
    fn = lib().hko_poly_loss_f64 if x.dtype == np.float64 else lib().hko_poly_loss_f32
    parallel(lambda bb, cc: fn(_p(x), _p(t), a, b, c, _p(r), bb, cc), n, threads)
    return r


def poly_loss_vjp_rows(x, t, bar_r, a, b, c, threads: int = 1):
    """``(hi, comp)`` of shape (3, rows): the 32-sample rows of the 3 Param gradients."""
    n = x.shape[0]
    rows = -(-n // 32)
    hi = np.empty((3, rows), dtype=x.dtype)
    comp = np.empty((3, rows), dtype=x.dtype)
    fn = lib().hko_poly_loss_vjp_rows_f64 if x.dtype == np.float64 else lib().hko_poly_loss_vjp_rows_f32

    def tile(r0, nr):
        h = np.empty((3, nr), dtype=x.dtype)
        cc = np.empty((3, nr), dtype=x.dtype)
        fn(_p(x), _p(t), _p(bar_r), a, b, c, n, r0, nr, _p(h), _p(cc))
        hi[:, r0:r0 + nr] = h
        comp[:, r0:r0 + nr] = cc

    parallel(tile, rows, threads)
    return hi, comp


def cells_finish(hi: np.ndarray, comp: np.ndarray | None, op: str = "sum"):
    hi = np.ascontiguousarray(hi)
    comp = None if comp is None else np.ascontiguousarray(comp)
    fn = lib().hko_cells_finish_f64 if hi.dtype == np.float64 else lib().hko_cells_finish_f32
    return fn(OP[op], _p(hi), None if comp is None else _p(comp), hi.shape[0])


def cells_leaves(hi: np.ndarray, comp: np.ndarray, op: str = "sum"):
    """The leaf partials ``(leaf_hi, leaf_comp)`` of float64 or float32 rows
    (4096 rows a leaf), in the rows' type."""
    hi, comp = np.ascontiguousarray(hi), np.ascontiguousarray(comp)
    leaves = -(-hi.shape[0] // 4096)
    lh, lc = np.empty(leaves, dtype=hi.dtype), np.empty(leaves, dtype=hi.dtype)
    fn = lib().hko_cells_leaves_d if hi.dtype == np.float64 else lib().hko_cells_leaves_f
    fn(OP[op], _p(hi), _p(comp), hi.shape[0], _p(lh), _p(lc))
    return lh, lc


def cells_tree(leaf_hi: np.ndarray, leaf_comp: np.ndarray, op: str = "sum") -> float:
    """The pairwise levels over leaf partials (float64 unless both are float32)."""
    f32 = np.asarray(leaf_hi).dtype == np.float32 and np.asarray(leaf_comp).dtype == np.float32
    dt = np.float32 if f32 else np.float64
    lh, lc = np.array(leaf_hi, dtype=dt), np.array(leaf_comp, dtype=dt)
    fn = lib().hko_cells_tree_f if f32 else lib().hko_cells_tree_d
    return fn(OP[op], _p(lh), _p(lc), lh.shape[0])


def cells_tree_pair(leaf_hi: np.ndarray, leaf_comp: np.ndarray, op: str = "sum") -> tuple:
    """The tree's root (hi, comp) pair before its final rounding (the compacting
    levels leave it at index 0)."""
    lh, lc = np.array(leaf_hi, dtype=np.float64), np.array(leaf_comp, dtype=np.float64)
    lib().hko_cells_tree_d(OP[op], _p(lh), _p(lc), lh.shape[0])
    return float(lh[0]), float(lc[0])


def poly_loss_vjp(x, t, bar_r, a, b, c, threads: int = 1):
    """The three Param gradients (cells) and the rows they were finished from."""
    hi, comp = poly_loss_vjp_rows(x, t, bar_r, a, b, c, threads)
    cells = [cells_finish(hi[k], comp[k]) for k in range(3)]
    return cells, (hi, comp)


def gravity(r1, r2, m1, m2, G, threads: int = 1):
    n = r1.shape[-1]
    f = np.empty_like(r1)
    u = np.empty(n)
    parallel(lambda b, c: lib().hko_gravity(_p(r1), _p(r2), n, _p(m1), _p(m2), G, _p(f), n, _p(u), b, c),
             n, threads)
    return f, u


def gravity_jvp(r1, r2, dr1, dr2, m1, m2, G, threads: int = 1):
    n = r1.shape[-1]
    df = np.empty_like(r1)
    du = np.empty(n)
    parallel(lambda b, c: lib().hko_gravity_jvp(_p(r1), _p(r2), _p(dr1), _p(dr2), n, _p(m1), _p(m2), G,
                                               _p(df), n, _p(du), b, c), n, threads)
    return df, du


def gravity_vjp(r1, r2, bar_f, bar_u, m1, m2, G, threads: int = 1):
    n = r1.shape[-1]
    b1 = np.empty_like(r1)
    b2 = np.empty_like(r1)
    parallel(lambda b, c: lib().hko_gravity_vjp(_p(r1), _p(r2), _p(bar_f), n, _p(bar_u), _p(m1), _p(m2), G,
                                               _p(b1), _p(b2), n, b, c), n, threads)
    return b1, b2


def spd_solve(A, b, threads: int = 1):
    n = A.shape[-1]
    x = np.empty_like(b)
    parallel(lambda bb, c: lib().hko_spd_solve(_p(A), _p(b), n, _p(x), n, bb, c), n, threads)
    return x


def spd_solve_vjp(A, b, bar_x, threads: int = 1):
    n = A.shape[-1]
    bar_A = np.empty_like(A)
    bar_b = np.empty_like(b)
    parallel(lambda bb, c: lib().hko_spd_solve_vjp(_p(A), _p(b), _p(bar_x), n, _p(bar_A), _p(bar_b), n, bb, c),
             n, threads)
    return bar_A, bar_b


OPS = {"sum": 0, "max": 1, "min": 2}


def rows(terms, op: str = "sum"):
    """``(hi, comp)``: the 32-sample rows of one column of terms, as the host
    frame makes them (float64)."""
    terms = np.ascontiguousarray(terms, dtype=np.float64)
    n = terms.shape[0]
    nrows = -(-n // 32)
    hi, comp = np.empty(max(nrows, 1)), np.empty(max(nrows, 1))
    lib().hko_rows_f64(OPS[op], _p(terms), n, _p(hi), _p(comp))
    return hi[:nrows], comp[:nrows]


def banded_rows(terms, op: str = "sum"):
    """The banded mode's rows of one column: each row's compensated pair
    rounded once (hi + comp) and a zero companion; max/min rows as they are."""
    hi, comp = rows(terms, op)
    if op != "sum":
        return hi, np.zeros_like(hi)
    return hi + comp, np.zeros_like(hi)


def sample_sum(terms, op: str = "sum") -> float:
    """A reduction over samples as a kernel makes it: the 32-sample rows of
    the terms, then the ordered finish of the rows into the cell."""
    terms = np.ascontiguousarray(terms, dtype=np.float64)
    n = terms.shape[0]
    rows = -(-n // 32)
    hi, comp = np.empty(max(rows, 1)), np.empty(max(rows, 1))
    lib().hko_rows_f64(OPS[op], _p(terms), n, _p(hi), _p(comp))
    return float(lib().hko_cells_finish_f64(OPS[op], _p(hi), _p(comp), rows))


def share(x):
    """z = x / sum(x)."""
    return x / sample_sum(x)


def standard(x):
    """mu = mean(x); v = mean((x - mu)^2); z = (x - mu) / sqrt(v); t = sum(z^2):
    the stages' bodies, each a mean as the sum of x_i / n."""
    n = float(x.shape[0])
    mu = sample_sum(x / n)
    d = x - mu
    v = sample_sum((d * d) / n)
    z = (x - mu) / np.sqrt(v)
    t = sample_sum(z * z)
    return mu, z, t


def centred(x):
    """v = (x, x^2, 2x); z = v - mean(v) per component (a vector divided by the
    count is multiplied by its reciprocal)."""
    n = x.shape[0]
    v = np.stack([x, x * x, 2.0 * x])
    r = 1.0 / float(n)
    mean = np.array([sample_sum(v[k] * r) for k in range(3)])
    return v - mean[:, None]


def team_chol(A, b, B, threads: int = 1):
    """(x, X, L, info) of the team-form Cholesky kernel: A (n, n, N), b (n, N), B (n, 2, N)."""
    k, n = A.shape[0], A.shape[-1]
    x, X, L = np.empty((k, n)), np.empty((k, 2, n)), np.empty((k, k, n))
    info = np.empty(n, dtype=np.int32)
    parallel(lambda bb, c: lib().hko_team_chol(k, _p(A), _p(b), _p(B), n, _p(x), _p(X), _p(L), _p(info), bb, c),
             n, threads)
    return x, X, L, info


def team_lu(A, b, B, threads: int = 1):
    """(x, X, det, info) of the team-form LU kernel."""
    k, n = A.shape[0], A.shape[-1]
    x, X, det = np.empty((k, n)), np.empty((k, 2, n)), np.empty(n)
    info = np.empty(n, dtype=np.int32)
    parallel(lambda bb, c: lib().hko_team_lu(k, _p(A), _p(b), _p(B), n, _p(x), _p(X), _p(det), _p(info), bb, c),
             n, threads)
    return x, X, det, info


def team_chol_from(A, b, threads: int = 1):
    """(x, L, info) of the chol_from kernel."""
    k, n = A.shape[0], A.shape[-1]
    x, L = np.empty((k, n)), np.empty((k, k, n))
    info = np.empty(n, dtype=np.int32)
    parallel(lambda bb, c: lib().hko_team_chol_from(k, _p(A), _p(b), n, _p(x), _p(L), _p(info), bb, c), n, threads)
    return x, L, info


def kepler(e, M, threads: int = 1):
    n = e.shape[0]
    E = np.empty(n)
    it = np.empty(n, dtype=np.int32)
    parallel(lambda b, c: lib().hko_kepler(_p(e), _p(M), _p(E), _p(it), b, c), n, threads)
    return E, it


def trig(x, threads: int = 1):
    """(sin x, cos x) by the host's libm."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    n = x.shape[0]
    s, c = np.empty(n), np.empty(n)
    parallel(lambda b, cc: lib().hko_trig(_p(x), _p(s), _p(c), b, cc), n, threads)
    return s, c


def kepler_vjp(e, M, bar_E, threads: int = 1):
    n = e.shape[0]
    be = np.empty(n)
    bM = np.empty(n)
    parallel(lambda b, c: lib().hko_kepler_vjp(_p(e), _p(M), _p(bar_E), _p(be), _p(bM), b, c), n, threads)
    return be, bM


# ------------------------------------------------------------- stepping kernels
def _stepped(fn, n: int, threads: int) -> int:
    counts = []
    lock = threading.Lock()

    def tile(b, c):
        got = fn(b, c)
        with lock:
            counts.append(int(got))

    parallel(tile, n, threads)
    return sum(counts)


def oscillator(planes: dict, dt: float, word: int, threads: int = 1) -> int:
    """One launch of the automatic RK4 oscillator with the fused_steps ``word``,
    in place on ``planes`` (x, v, k, nstop, omega, zeta float64; terminated
    uint8/bool); returns the samples it newly finished."""
    x, v, k = planes["x"], planes["v"], planes["k"]
    term = planes["terminated"].view(np.uint8)
    n = x.shape[0]
    return _stepped(lambda b, c: lib().hko_oscillator(_p(x), _p(v), _p(k), _p(planes["nstop"]), _p(planes["omega"]),
                                                      _p(planes["zeta"]), _p(term), float(dt), int(word), b, c),
                    n, threads)


def orbit(planes: dict, word: int, threads: int = 1) -> int:
    """One launch of the automatic Fehlberg 7(8) orbit kernel with ``word``, in
    place on ``planes`` (s (6, n), t, h, n_acc, n_rej, t_end float64;
    terminated); returns the samples it newly finished."""
    s = planes["s"]
    term = planes["terminated"].view(np.uint8)
    n = s.shape[1]
    return _stepped(lambda b, c: lib().hko_orbit(_p(s), n, _p(planes["t"]), _p(planes["h"]), _p(planes["n_acc"]),
                                                 _p(planes["n_rej"]), _p(planes["t_end"]), _p(term), int(word), b, c),
                    n, threads)


def share_vjp(x, bar_z):
    """The VJP of share wrt x, as its stages compute it: S = sum(x),
    c = sum(-((bar_z (x / S)) / S)), bar_x = bar_z / S + c."""
    s = sample_sum(x)
    c = sample_sum(-((bar_z * (x / s)) / s))
    return (bar_z / s) + c


def key_sums(x, rows: int = 8):
    """Per key (``rows`` consecutive lanes), the sum an aligned-run commit makes
    on a fully converged warp: the xor butterfly over the run's lanes (offsets
    rows / 2, ..., 1; lane l adds lane l ^ o), then one add into the zeroed slot
    (hk/accum.cuh groups)."""
    v = np.ascontiguousarray(x, dtype=np.float64).reshape(-1, rows).copy()
    o = rows // 2
    while o >= 1:
        idx = np.arange(rows) ^ o
        v = v + v[:, idx]
        o //= 2
    return 0.0 + v[:, 0]


def key_share(x, rows: int = 8):
    """z = x / (its key's sum)."""
    s = key_sums(x, rows)
    return x / np.repeat(s, rows)


def block_sums(u, v=None, rows: int = 8):
    """Per key (``rows`` consecutive lanes), the block sum_r u[:, r] v[:, r]^T
    in lane order from 0 (a BlockSum team stage): ``u`` is (p, lanes), ``v``
    (q, lanes) or None for the constant 1; the result is (p, q, keys), or
    (p, keys) when ``v`` is None."""
    u = np.asarray(u, dtype=np.float64)
    p, lanes = u.shape
    keys = lanes // rows
    uu = u.reshape(p, keys, rows)
    if v is None:
        s = np.zeros((p, keys))
        for r in range(rows):
            s = s + uu[:, :, r]
        return s
    v = np.asarray(v, dtype=np.float64)
    vv = v.reshape(v.shape[0], keys, rows)
    s = np.zeros((p, v.shape[0], keys))
    for r in range(rows):
        s = s + (uu[:, None, :, r] * vv[None, :, :, r])
    return s


#: The ordered sum's fixed grouping (hawk/emit/team.py:208-240; the numpy
#: emulation the reference's tests hold it to, tests/test_ordered_fixed_tree.py:21-40).
ORDERED_VIRTUAL, ORDERED_GROUPS, ORDERED_GROUP_LANES = 65536, 64, 1024


def _halving(s):
    """The halving tree s[i] += s[i + w], w = len/2 ... 1, over the last axis."""
    w = s.shape[-1] // 2
    while w:
        s = s[..., :w] + s[..., w:2 * w]
        w //= 2
    return s[..., 0]


def ordered_sums(x, rows: int):
    """Per key (``rows`` consecutive lanes), the ordered sum: virtual lane l
    of 65536 adds rows l, l + 65536, ... in order from 0; each group of 1024
    virtual lanes folds by the halving tree (the first stage), the 64 group
    values by the same tree (the second).  Zero padding adds exactly: a sum
    started at +0 is never -0 under round to nearest."""
    v = np.ascontiguousarray(x, dtype=np.float64).reshape(-1, rows)
    part = np.zeros((v.shape[0], ORDERED_VIRTUAL))
    for r in range(0, rows, ORDERED_VIRTUAL):
        blk = v[:, r:r + ORDERED_VIRTUAL]
        part[:, :blk.shape[1]] += blk
    groups = _halving(part.reshape(v.shape[0], ORDERED_GROUPS, ORDERED_GROUP_LANES))
    return _halving(groups)


def ordered_scatter(key, x, acc):
    """``hawk.scatter(acc, policy="ordered")[key] += x`` as the reference's
    stages fold it (hawk/ir/team.py:716-736; hawk/emit/team.py:322-460):
    chunks = clamp(n // cells, 1, 256) runs of ceil(n / chunks) lanes; each
    chunk sums its lanes' values per cell in lane order from 0; each cell adds
    its chunks' sums in chunk order from 0 and then adds that onto ``acc``.
    Key -1 is skipped; any other key outside [0, cells) is dropped and
    reported.  Returns (acc after the run, whether a key was reported)."""
    key = np.asarray(key, dtype=np.int64)
    x = np.asarray(x, dtype=np.float64)
    acc = np.array(acc, dtype=np.float64, copy=True)
    n, cells = key.shape[0], acc.shape[0]
    chunks = min(256, max(1, n // max(cells, 1)))
    span = -(-n // chunks) if n else 0
    pad = chunks * span - n
    k = np.concatenate([key, np.full(pad, -1)]).reshape(chunks, span)
    v = np.concatenate([x, np.zeros(pad)]).reshape(chunks, span)
    good = (k >= 0) & (k < cells)
    bad = bool(np.any(~good & (k != -1)))
    part = np.zeros((cells + 1, chunks))     # row ``cells`` takes the dropped lanes
    c = np.arange(chunks)
    for t in range(span):
        tgt = np.where(good[:, t], k[:, t], cells)
        part[tgt, c] += v[:, t]
    s = np.zeros(cells)
    for b in range(chunks):
        s = s + part[:cells, b]
    return acc + s, bad


def net_axis(w, x, y, mask):
    """Per-net loss and its gradient wrt the weights, by numpy over the nets
    (the reference's loop, tests/test_net_axis.py:61-73): ``w`` (K, 24) holds
    (a, b, c) per hidden unit, ``x``/``y`` (K, S), ``mask`` (K, 8);
    t = tanh(a x + b), r = (mask c) . t - y, loss = r . r."""
    w, x, y, mask = (np.asarray(v, dtype=np.float64) for v in (w, x, y, mask))
    a, b, c = w[:, 0::3], w[:, 1::3], w[:, 2::3]
    t = np.tanh(a[:, :, None] * x[:, None, :] + b[:, :, None])
    r = np.einsum("kh,khs->ks", mask * c, t) - y
    loss = np.einsum("ks,ks->k", r, r)
    grad = np.zeros_like(w)
    dt = (2 * mask * c)[:, :, None] * (1 - t * t) * r[:, None, :]
    grad[:, 0::3] = np.einsum("khs,ks->kh", dt, x)
    grad[:, 1::3] = dt.sum(axis=2)
    grad[:, 2::3] = np.einsum("khs,ks->kh", (2 * mask)[:, :, None] * t, r)
    return loss, grad


def sym_eigen(A, vectors: bool = True, threads: int = 1):
    """(w, V, info) of eigh(A) per sample (V None for the values-only kernel)."""
    k, n = A.shape[0], A.shape[-1]
    w = np.empty((k, n))
    V = np.empty((k, k, n)) if vectors else None
    info = np.empty(n, dtype=np.int32)
    parallel(lambda b, c: lib().hko_sym_eigen(k, _p(A), n, _p(w), _p(V) if V is not None else None, _p(info), b, c),
             n, threads)
    return w, V, info


def lstsq_qr(J, r, threads: int = 1):
    """(x, info) of lstsq(J, r) per sample by the team-form Householder QR."""
    m, n, lanes = J.shape
    x = np.empty((n, lanes))
    info = np.empty(lanes, dtype=np.int32)
    parallel(lambda b, c: lib().hko_lstsq_qr(m, n, _p(J), _p(r), lanes, _p(x), _p(info), b, c), lanes, threads)
    return x, info
