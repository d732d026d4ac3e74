"""Make the golden vectors the oracle is pinned against.

Every kernel of ``hawk_b200.configs`` (fwd, VJP, JVP) is evaluated sample by
sample by the reference's own numpy IR interpreter -- ``evaluate`` in the
reference's tests/_eval.py:264, "deliberately naive ... independent of the
emitter" -- on seeded inputs drawn by ``hawk_b200.workloads``, and the inputs
and outputs are written to ``tests/golden/<config>.npz``.  The VJP of the
affine polynomial is evaluated on its un-promoted form (Params by value), which
gives the per-sample gradient terms the 32-sample rows sum.

Needs the reference checkout (its front end and tests/ directory); the
fixtures it writes are committed and are all the test suite reads.

    python tests/golden/make_golden.py          # every fixture
    python tests/golden/make_golden.py team     # the team-form fixtures only
    python tests/golden/make_golden.py eigen    # the symmetric-eigenproblem fixtures only
    python tests/golden/make_golden.py ordered  # the ordered-sum fixtures only
    python tests/golden/make_golden.py net      # the net-axis fixtures only
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

N = {"energy": 96, "poly_loss": 160, "gravity": 96, "spd_solve": 48, "kepler": 128}
SEED = 20261201
#: fused_steps words of the stepping fixtures (1: the single step; 0 and a
#: negative word run no trip; the rest run up to that many).
OSC_WORDS = (1, 0, -2, 5, 30)
ORB_WORDS = (1, 9, 40)


#: Team-form fixtures: (kernel, workload kind, n, lanes); lane TEAM_BAD fails.
TEAM_CASES = (("team_chol", "spd", 33, 5), ("team_lu", "general", 33, 5), ("team_chol", "spd", 64, 3),
              ("team_chol_from", "lower", 64, 3))


def team_fixtures(evaluate) -> None:
    """team.npz: the team-form kernels' inputs and the interpreter's outputs
    (its linear algebra is scipy's LAPACK, so these pin the oracle within the
    reference's tolerances, and the status words exactly)."""
    from hawk_b200 import configs, workloads

    out = {}
    for kernel, kind, n, lanes in TEAM_CASES:
        name = f"{kernel}_{n}"
        k = configs.TEAM_KERNELS[name]
        w = workloads.team(n, lanes, kind, SEED + n)
        outs = [o for r, o in k.walk.arg_spec if r == "mutable"]
        got = {o: [] for o in outs}
        for i in range(lanes):
            env = {"A": w["A"][..., i], "b": w["b"][:, i], "B": w["B"][..., i]}
            res = evaluate(k.sinks, env)
            for o in outs:
                got[o].append(np.asarray(res[o], dtype=np.int32 if o == "info" else float))
        for key in ("A", "b", "B"):
            out[f"{name}_{key}"] = w[key]
        for o in outs:
            out[f"{name}_{o}"] = np.stack(got[o], axis=-1)
    np.savez(HERE / "team.npz", **out)


def eigen_fixtures(evaluate) -> None:
    """eigen.npz: symmetric 6 x 6 matrices (lane 2: a repeated eigenvalue) and
    the interpreter's eigh (numpy's, signed so each vector's largest component
    is positive)."""
    from hawk_b200 import configs

    rng = np.random.default_rng(SEED)
    lanes, n = 6, 6
    mats = []
    for lane in range(lanes):
        g = rng.standard_normal((n, n))
        a = (g + g.T) / 2
        if lane == 2:
            q, _ = np.linalg.qr(rng.standard_normal((n, n)))
            a = (q * np.r_[np.ones(n // 2), np.linspace(2, 3, n - n // 2)]) @ q.T
        mats.append(a)
    A = np.ascontiguousarray(np.moveaxis(np.stack(mats), 0, -1))
    outs = {"w": [], "V": [], "info": []}
    for i in range(lanes):
        res = evaluate(configs.sym_eigen.sinks, {"A": A[..., i]})
        for k in outs:
            outs[k].append(np.asarray(res[k], dtype=np.int32 if k == "info" else float))
    np.savez(HERE / "eigen.npz", A=A, **{k: np.stack(v, axis=-1) for k, v in outs.items()})


#: Ordered-sum fixtures: keys of ``rows`` lanes, drawn as the reference's
#: fixed-tree test draws them (normal times exp(normal), seeded by the count).
ORDERED_ROWS = ((8, 5), (1, 3), (1000, 2), (65536, 1), (197385, 2), (200003, 1))


def ordered_draw(rows: int, keys: int) -> np.ndarray:
    n = rows * keys
    return np.random.default_rng(n).normal(size=n) * np.exp(np.random.default_rng(n + 1).normal(size=n))


def ordered_fixtures(tree_sum) -> None:
    """ordered.npz: per (rows, keys) case, each key's ordered sum by the
    reference's own numpy emulation of the fixed grouping (``tree_sum``,
    tests/test_ordered_fixed_tree.py:33-40 in the reference) and a digest of
    the drawn lanes (the fixture keeps the seed, not the lanes)."""
    import hashlib

    out = {}
    for rows, keys in ORDERED_ROWS:
        x = ordered_draw(rows, keys)
        out[f"sum_{rows}_{keys}"] = np.array([tree_sum(x[k * rows:(k + 1) * rows]) for k in range(keys)])
        out[f"sha_{rows}_{keys}"] = np.frombuffer(hashlib.sha256(x.tobytes()).digest(), np.uint8)
    np.savez(HERE / "ordered.npz", **out)


def net_fixtures(problem, loop) -> None:
    """net.npz: five nets of widths (8, 3, 5, 1, 6) at 40 and 48 samples, drawn
    by the reference's ``_problem`` and solved by its loop over the nets
    (``_oracle``, tests/test_net_axis.py:52-73 in the reference)."""
    out = {}
    for s in (40, 48):
        w, x, y, mask = problem(5, (8, 3, 5, 1, 6), seed=3, S=s)
        loss, grad = loop(w, x, y, mask)
        out.update({f"w_{s}": w, f"x_{s}": x, f"y_{s}": y, f"mask_{s}": mask, f"loss_{s}": loss, f"grad_{s}": grad})
    np.savez(HERE / "net.npz", **out)


def main() -> int:
    from hawk_b200 import frontend, workloads

    if sys.argv[1:] == ["net"]:
        hawk = frontend.load()
        sys.path.insert(0, str(Path(hawk.__file__).resolve().parent.parent / "tests"))
        from test_net_axis import _oracle, _problem
        net_fixtures(_problem, _oracle)
        return 0

    if sys.argv[1:] == ["ordered"]:
        hawk = frontend.load()
        sys.path.insert(0, str(Path(hawk.__file__).resolve().parent.parent / "tests"))
        from test_ordered_fixed_tree import tree_sum
        ordered_fixtures(tree_sum)
        return 0

    if sys.argv[1:] == ["eigen"]:
        hawk = frontend.load()
        sys.path.insert(0, str(Path(hawk.__file__).resolve().parent.parent / "tests"))
        from _eval import evaluate
        eigen_fixtures(evaluate)
        return 0

    if sys.argv[1:] == ["team"]:
        hawk = frontend.load()
        sys.path.insert(0, str(Path(hawk.__file__).resolve().parent.parent / "tests"))
        from _eval import evaluate
        team_fixtures(evaluate)
        return 0

    hawk = frontend.load()
    root = Path(hawk.__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "tests"))
    from _eval import evaluate  # the reference's IR interpreter

    from hawk import Kernel
    from hawk.diff import jvp, vjp

    from hawk_b200 import configs

    def per_sample(kernel_sinks, envs, names):
        out = {k: [] for k in names}
        for env in envs:
            got = evaluate(kernel_sinks, env)
            for k in names:
                out[k].append(np.asarray(got[k], dtype=float))
        return {k: np.stack(v, axis=-1) for k, v in out.items()}

    # c1 energy
    w = workloads.energy(N["energy"], SEED)
    envs = [{"v": w["v"][:, i], "bar_out": w["bar_out"][i], "dot_v": w["dot_v"][:, i]} for i in range(N["energy"])]
    g = {}
    g.update({"out": per_sample(configs.energy.sinks, envs, ["out"])["out"]})
    g.update({"bar_v": per_sample(configs.KERNELS["energy_vjp"][0].sinks, envs, ["bar_v"])["bar_v"]})
    g.update({"dot_out": per_sample(configs.KERNELS["energy_jvp"][0].sinks, envs, ["dot_out"])["dot_out"]})
    np.savez(HERE / "energy.npz", v=w["v"], bar_out=w["bar_out"], dot_v=w["dot_v"], **g)

    # c2 affine polynomial (and the per-sample terms of its Param VJP)
    w = workloads.poly_loss(N["poly_loss"], SEED)
    plain_vjp = vjp(configs.poly_loss, wrt=("a", "b", "c"))
    envs = [{"x": w["x"][i], "t": w["t"][i], "a": w["a"], "b": w["b"], "c": w["c"], "bar_r": w["bar_r"][i]}
            for i in range(N["poly_loss"])]
    r = per_sample(configs.poly_loss.sinks, envs, ["r"])["r"]
    terms = per_sample(plain_vjp, envs, ["bar_a", "bar_b", "bar_c"])
    np.savez(HERE / "poly_loss.npz", x=w["x"], t=w["t"], bar_r=w["bar_r"], a=w["a"], b=w["b"], c=w["c"], r=r,
             term_a=terms["bar_a"], term_b=terms["bar_b"], term_c=terms["bar_c"])

    # c3 gravity
    w = workloads.gravity(N["gravity"], SEED)
    envs = [{"r1": w["r1"][:, i], "r2": w["r2"][:, i], "m1": w["m1"][i], "m2": w["m2"][i], "G": w["G"],
             "dot_r1": w["dr1"][:, i], "dot_r2": w["dr2"][:, i], "bar_f": w["bar_f"][:, i],
             "bar_u": w["bar_u"][i]} for i in range(N["gravity"])]
    fwd = per_sample(configs.gravity.sinks, envs, ["f", "u"])
    tan = per_sample(configs.KERNELS["gravity_jvp"][0].sinks, envs, ["dot_f", "dot_u"])
    adj = per_sample(configs.KERNELS["gravity_vjp"][0].sinks, envs, ["bar_r1", "bar_r2"])
    np.savez(HERE / "gravity.npz", **{k: w[k] for k in ("r1", "r2", "m1", "m2", "dr1", "dr2", "bar_f", "bar_u")},
             G=w["G"], **fwd, **tan, **adj)

    # c4 SPD solve
    w = workloads.spd_solve(N["spd_solve"], SEED)
    envs = [{"A": w["A"][:, :, i], "b": w["b"][:, i], "bar_x": w["bar_x"][:, i]} for i in range(N["spd_solve"])]
    fwd = per_sample(configs.spd_solve.sinks, envs, ["x"])
    adj = per_sample(configs.KERNELS["spd_solve_vjp"][0].sinks, envs, ["bar_A", "bar_b"])
    np.savez(HERE / "spd_solve.npz", A=w["A"], b=w["b"], bar_x=w["bar_x"], **fwd, **adj)

    # c5 Kepler
    w = workloads.kepler(N["kepler"], SEED)
    envs = [{"e": w["e"][i], "M": w["M"][i], "bar_E": w["bar_E"][i]} for i in range(N["kepler"])]
    fwd = per_sample(configs.kepler.sinks, envs, ["E", "iters"])
    adj = per_sample(configs.KERNELS["kepler_vjp"][0].sinks, envs, ["bar_e", "bar_M"])
    # the reference's known answer: e = 0.5, M = 1.0
    known = evaluate(configs.kepler.sinks, {"e": 0.5, "M": 1.0, "bar_E": 1.0})
    np.savez(HERE / "kepler.npz", e=w["e"], M=w["M"], bar_E=w["bar_E"], E=fwd["E"],
             iters=fwd["iters"].astype(np.int32), bar_e=adj["bar_e"], bar_M=adj["bar_M"],
             known_E=float(known["E"]), known_iters=int(known["iters"]))
    # the ordered finish of rows into a cell (the reference's hawk/_cells.py:94-119)
    from hawk import _cells

    rng = np.random.default_rng(SEED)
    cells = {}
    for n in (1, 2, 31, 255, 256, 257, 4095, 4096, 4097, 12289, 16385):
        hi = rng.standard_normal(n) * np.exp(rng.uniform(-20, 20, n))
        comp = rng.standard_normal(n) * np.abs(hi) * 1e-17
        cells[f"hi_{n}"] = hi
        cells[f"comp_{n}"] = comp
        for op in ("sum", "max", "min"):
            cells[f"{op}_{n}"] = np.float64(_cells.finish(hi, comp, op))
        cells[f"sum32_{n}"] = np.float32(_cells.finish(hi.astype(np.float32), comp.astype(np.float32), "sum"))
    np.savez(HERE / "cells.npz", **cells)

    # s1/s2 automatic stepping kernels: one launch per fused_steps word, each
    # sample evaluated from the same start (the interpreter runs the fused
    # loop's trips; word 1 is the single step).  Samples finished on entry are
    # left out: the mask guard is the entry's, not the IR's.
    steps = {}
    w = workloads.oscillator(48, SEED, stop_max=24)
    osc = configs.KERNELS["oscillator"][0]
    steps.update({f"osc_{k}": (np.asarray(v) if k != "dt" else np.float64(v)) for k, v in w.items()})
    for word in OSC_WORDS:
        sinks = osc.one_step.sinks if word == 1 else osc.sinks
        envs = [{**{k: w[k][i] for k in ("omega", "zeta", "nstop", "x", "v", "k")}, "dt": w["dt"],
                 "terminated": False, "fused_steps": np.array([word]),
                 "finished_count": np.array([0], dtype=np.uint32)} for i in range(48)]
        got = per_sample(sinks, envs, ["x", "v", "k", "terminated"])
        for k in ("x", "v", "k", "terminated"):
            steps[f"osc_w{word}_{k}"] = got[k]
    w = workloads.orbit(12, SEED)
    orb = configs.KERNELS["orbit"][0]
    steps.update({f"orb_{k}": np.asarray(v) for k, v in w.items()})
    for word in ORB_WORDS:
        sinks = orb.one_step.sinks if word == 1 else orb.sinks
        envs = [{"s": w["s"][:, i], **{k: w[k][i] for k in ("t", "h", "n_acc", "n_rej", "t_end")},
                 "terminated": False, "fused_steps": np.array([word]),
                 "finished_count": np.array([0], dtype=np.uint32)} for i in range(12)]
        got = per_sample(sinks, envs, ["s", "t", "h", "n_acc", "n_rej", "terminated"])
        for k in ("s", "t", "h", "n_acc", "n_rej", "terminated"):
            steps[f"orb_w{word}_{k}"] = got[k]
    np.savez(HERE / "steps.npz", **steps)
    team_fixtures(evaluate)
    eigen_fixtures(evaluate)
    _ = Kernel, jvp
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
