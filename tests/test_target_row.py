"""The b200 row as a drop-in target of the reference's build (no GPU).

* The row's ``features`` are exactly what the b200 build makes: one planted
  kernel per entry of the reference's feature table
  (hawk/targets/features.py:74-152) either renders and compiles for sm_100a
  (the features the row lists) or is refused by name, with the reference's
  reason and alternative (the way the reference's C row refuses,
  tests/test_embedded_refusals.py).
* The reference's own ``hawk.build(..., targets=("b200",))``
  (hawk/artifact/bundle.py:1349), with the b200 branches of its render and
  compile seams wired in (``hawk_b200.target.seams``), writes units
  byte-identical to the committed bundles, the same ``b200`` sidecar block,
  CUBINs equal to a fresh compile, and its own manifest.
* Every committed unit re-renders byte for byte from the kernels.

Needs the reference's front end and NVRTC (cuda-python); skipped without them.
"""

from __future__ import annotations

import json
import tempfile
from pathlib import Path

import pytest

from conftest import REPO

try:
    from hawk_b200 import configs
    from hawk_b200.target.nvrtc import compile_cubin
    from cuda.bindings import nvrtc as _nvrtc  # noqa: F401
except Exception as exc:                                   # noqa: BLE001
    pytest.skip(f"the reference front end or NVRTC is not importable here ({exc})", allow_module_level=True)

import hawk  # noqa: E402  (brought up by hawk_b200.configs)
import hawk.math as hm  # noqa: E402
from hawk import Index, Mutable, Param, Scalar, Terminated, Vector  # noqa: E402
from hawk.emit import compose  # noqa: E402
from hawk.ext import Guard, Kind, sink_policy  # noqa: E402
from hawk.ir import Assign, Leaf  # noqa: E402
from hawk.ir.loop_nodes import Loop, LoopCarry, LoopIndex, LoopValue  # noqa: E402
from hawk.ir.nodes import AccumWrite, Const  # noqa: E402
from hawk.ir.ops import make  # noqa: E402
from hawk.targets import FEATURES  # noqa: E402
from hawk.trace.kernel import Kernel  # noqa: E402
from hawk.types import TensorType  # noqa: E402

from hawk_b200.errors import HawkError  # noqa: E402
from hawk_b200.target import install, row  # noqa: E402
from hawk_b200.target.assemble import BUILT_FEATURES  # noqa: E402
from hawk_b200.target.build import choose_unit  # noqa: E402
from hawk_b200.target.seams import wired  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
F64 = TensorType((), "f64")


# ------------------------------------------------------------ planted kernels
@hawk.kernel
def draws(seed: Index, counter: Index, y: Mutable[Scalar]):
    y = hm.random.normal(seed, counter)


_TWICE = hawk.raw_device("mut_y = 2.0 * psc_x;", access="sample_local", returns=Scalar)


@hawk.kernel
def raw_twice(x: Scalar, y: Mutable[Scalar]):
    y = _TWICE(x)


@hawk.kernel
def summed(v: Vector[3], total: Mutable[Scalar]):
    total = hawk.sum(hm.dot(v, v))


@hawk.kernel
def other_sample(x: Scalar, j: Index, y: Mutable[Scalar]):
    y = x.at(j)


@hawk.kernel(kind=Kind("row_active", guard=Guard(active_set=True)))
def active_rows(w: Scalar, dt: Param, terminated: Terminated, x: Mutable[Scalar]):
    x = x + dt * w


@hawk.kernel
def branches(k: Index, b0: Scalar, b1: Scalar, y: Mutable[Scalar]):
    y = hm.dispatch(k, [b0, b1], policy="segmented")


@hawk.kernel(kind=Kind("row_compensated", sink=sink_policy("compensated", into="acc_c")))
def compensated_scatter(x: Scalar, lane: Index, acc: Mutable[Scalar], acc_c: Mutable[Scalar]):
    hawk.scatter(acc, policy="plain")[lane] += x
    hawk.scatter(acc_c, policy="plain")[lane] += 0.0


@hawk.kernel
def lane_one(x: Scalar, p: Mutable[Scalar]):
    p = x * 3.0


@hawk.kernel
def lane_two(x: Scalar, q: Mutable[Scalar]):
    q = x - 1.0


@hawk.kernel(steps=1)
def march(dt: Param, t_end: Scalar, terminated: Terminated, x: Mutable[Scalar]):
    xn = x + dt
    x = xn
    terminated = xn >= t_end


@hawk.kernel
def int_hypot(a: Index, b: Index, y: Mutable[Index]):
    y = hm.hypot(a, b)


def vector_scatter():
    """A scattered accumulate of a Vector[3], as IR (the tracer itself refuses
    to write one)."""
    v = Leaf("vocab_read", "vec_in", "v", TensorType((3,), "f64"))
    lane = Leaf("vocab_read", "per_sample", "lane", TensorType((), "i64"))
    return Kernel("vector_scatter", (AccumWrite("acc", v, lane, TensorType((3,), "f64")),))


def zero_trips():
    """A loop of no trips, as IR (the tracer folds ``range(0)`` away)."""
    x = Leaf("vocab_read", "per_sample", "x", F64)
    carry = LoopCarry(0, 0, "s", F64)
    loop = Loop(LoopIndex(0, "k"), (carry,), (x,), (make("mul", (carry, Const(2.0, F64))),), start=0, stop=0, step=1)
    return Kernel("zero_trips", (Assign("y", LoopValue(loop, 0), F64),))


@hawk.kernel
def vector_select(v: Vector[3], y: Mutable[Vector[3]]):
    y = hm.where(v > 0.0, v, -v)


PLANTED = {
    "random": lambda: draws,
    "linalg": lambda: configs.spd_solve,
    "raw_device": lambda: raw_twice,
    "sample_reduction": lambda: summed,
    "cross_sample_at": lambda: other_sample,
    "active_set": lambda: active_rows,
    "segmented": lambda: branches,
    "compensated": lambda: compensated_scatter,
    "fused_lanes": lambda: compose([lane_one, lane_two], "fused"),
    "two_path": lambda: hawk.steps(march, "auto"),
    "int_libm": lambda: int_hypot,
    "scattered_tensor_accum": vector_scatter,
    "zero_trip_loop": zero_trips,
    "tensor_select_cond": lambda: vector_select,
}


def test_every_feature_has_a_planted_kernel():
    assert set(PLANTED) == set(FEATURES)


def test_the_row_declares_exactly_the_features_it_builds():
    r = row()
    assert r.features == BUILT_FEATURES
    assert BUILT_FEATURES <= set(FEATURES)
    install()
    assert hawk.targets.TARGETS["b200"].features == BUILT_FEATURES


@pytest.mark.parametrize("feature", list(FEATURES))
def test_a_feature_builds_or_is_refused_by_name(feature):
    kernel = PLANTED[feature]()
    if feature in BUILT_FEATURES:
        unit, cubin, _log, ptxas = choose_unit(kernel, kernel.name, "float64")
        assert cubin and unit.name in ptxas
    else:
        with pytest.raises(HawkError) as err:
            choose_unit(kernel, kernel.name, "float64")
        assert f"does not build the feature {feature!r}" in str(err.value)


def test_the_compensated_sink_policy_commits_its_correction():
    unit, _cubin, _log, _ptxas = choose_unit(compensated_scatter, "compensated_scatter", "float64")
    assert "hawk_abi::accum_add_compensated(aout_acc, aout_acc_c," in unit.text


def _b200_block(sidecar: dict) -> dict:
    return {k: v for k, v in sidecar["b200"].items() if k not in ("unit", "cubin")}


def test_the_reference_build_writes_b200_artifacts_through_the_seams(tmp_path):
    kernels = [configs.energy, configs.KERNELS["energy_vjp"][0], configs.spd_solve]
    with wired():
        bundle = hawk.build(kernels, tmp_path, targets=("b200",), cache_dir=tempfile.mkdtemp())
    manifest = json.loads((tmp_path / "manifest.json").read_text())
    assert [p["id"] for p in manifest["plugins"]] == ["energy", "energy_vjp", "spd_solve"]
    assert {p["format"] for p in manifest["plugins"]} == {"cubin"}
    assert bundle.manifest_path == tmp_path / "manifest.json"
    for name in ("energy", "energy_vjp", "spd_solve"):
        text = (tmp_path / f"{name}.cu").read_text()
        assert text == (BUNDLES / f"{name}.float64.cu").read_text()
        ours = json.loads((BUNDLES / f"{name}.float64.json").read_text())
        theirs = json.loads((tmp_path / f"{name}.json").read_text())
        assert _b200_block(theirs) == _b200_block(ours)
        assert theirs["b200"]["cubin"] == f"{name}.cubin"
        assert (tmp_path / f"{name}.cubin").read_bytes() == compile_cubin(text, name)[0]
        assert theirs["arg_spec"] == ours["arg_spec"] and theirs["digest"] == ours["digest"]


def test_the_runtime_finds_a_reference_built_sidecar(tmp_path):
    from hawk_b200.runtime import sidecar_path

    with wired():
        hawk.build([configs.energy], tmp_path, targets=("b200",), cache_dir=tempfile.mkdtemp())
    assert sidecar_path(tmp_path, "energy", "float64") == tmp_path / "energy.json"
    assert sidecar_path(tmp_path, "energy", "float32") is None
    assert sidecar_path(BUNDLES, "energy", "float64") == BUNDLES / "energy.float64.json"


def _committed():
    out = []
    for name, (kernel, modes) in configs.KERNELS.items():
        for mode in modes:
            out.append((name, mode, False))
    out += [(name, "float64", True) for name in ("spd_solve_vjp", "poly_loss_vjp")]
    return out


@pytest.mark.parametrize("name,mode,staged", _committed(),
                         ids=[f"{n}.{m}{'.staged' if s else ''}" for n, m, s in _committed()])
def test_every_committed_unit_re_renders_byte_for_byte(name, mode, staged):
    from hawk_b200.target.build import build_kernel

    kernel, _modes = configs.KERNELS[name]
    with tempfile.TemporaryDirectory() as d:
        build_kernel(kernel, d, name=name, mode=mode, staged=True if staged else None)
        got = (Path(d) / f"{name}.{mode}.cu").read_text()
    committed = (BUNDLES / ("staged" if staged else "") / f"{name}.{mode}.cu").read_text()
    assert got == committed


@hawk.kernel
def banded_scatter(x: Scalar, lane: Index, acc: Mutable[Scalar]):
    hawk.scatter(acc)[lane] += x


@hawk.kernel
def banded_erf(x: Scalar, y: Mutable[Scalar]):
    y = hm.erf(x)


@pytest.mark.parametrize("kernel,what", [(banded_scatter, "scattered commit"), (banded_erf, "hawk.math.erf")],
                         ids=["scatter", "erf"])
def test_the_banded_mode_refuses_what_it_does_not_build(kernel, what):
    with pytest.raises(HawkError, match=what):
        choose_unit(kernel, kernel.name, "banded")
    choose_unit(kernel, kernel.name, "float64")


def test_a_banded_row_is_its_compensated_pair_rounded_once():
    unit, _cubin, _log, _ptxas = choose_unit(configs.band_rows, "band_rows", "banded")
    assert "aout_s.data()[hawk_row] = hawk_s + hawk_c;" in unit.text
    assert "aout_s_comp.data()[hawk_row] = static_cast<decltype(hawk_c)>(0);" in unit.text
    f64, _cubin, _log, _ptxas = choose_unit(configs.band_rows, "band_rows", "float64")
    assert "aout_s.data()[hawk_row] = hawk_s;" in f64.text
