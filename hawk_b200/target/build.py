"""Build b200 bundles: unit text, CUBIN and sidecar per kernel and scalar mode.

The b200 counterpart of the reference's ``build_bundle``
(hawk/artifact/bundle.py:1349) for one row: for each kernel it renders the
unit (``assemble.render_unit``), compiles it with NVRTC at sm_100a, and writes

* ``<name>.<mode>.cu``   the unit text (what was compiled),
* ``<name>.<mode>.cubin`` the sm_100a image the runtime loads,
* ``<name>.<mode>.json`` the sidecar: the reference's v2 sidecar fields the
  runtime binds from (``arg_spec``, ``arg_shapes``, ``arg_dtypes``,
  ``mutables``, ``vec_widths``, ``mat_shapes``, ``params``, ``param_planes``,
  ``accum_outputs``, ``digest`` ..., hawk/artifact/sidecar.py:348-486) plus a
  ``b200`` block (entry, frame, sample sums, arch, NVRTC options, ptxas report).
"""

from __future__ import annotations

import json
from pathlib import Path

from ..errors import HawkError
from .assemble import render_unit
from .nvrtc import ARCH, compile_cubin, options


def _reference_sidecar(name: str, walk, mode: str, lane_space=None) -> dict:
    """The reference's v2 sidecar for the kernel (its own function), or the
    subset this runtime reads when that function needs the reference's
    third-party packages.  ``lane_space`` is the kernel's launch shape
    (``Grid`` axes; the reference's sidecar records it as launch.lane_space)."""
    from unittest import mock

    try:
        from hawk.artifact import sidecar as sc

        extra = {} if lane_space is None else {"lane_space": lane_space}
        # The reference records where its third-party headers came from; a b200
        # unit includes only this build's device library, so that is recorded.
        with mock.patch.object(sc, "_root_or_sealed_marker", lambda resolver: "hawk_b200/csrc/include"):
            return sc.sidecar_meta(name, walk, fmt="cubin", scalar_type=mode, exec_targets=("device",), **extra)
    except Exception:                                   # noqa: BLE001 -- fall back to the read subset
        return _subset_sidecar(name, walk, mode)


def _subset_sidecar(name: str, walk, mode: str) -> dict:
    from hawk.artifact import sidecar as sc

    return {
        "format": "cubin",
        "kernel": name,
        "scalar_type": mode,
        "arg_spec": [list(p) for p in walk.arg_spec],
        "arg_shapes": sc._arg_shapes(walk),
        "arg_dtypes": sc._arg_dtypes(walk, mode),
        "mutables": sc._mutables(walk),
        "vec_widths": {n: int(walk.slot_types[("vec_in", n)].shape[0])
                       for r, n in walk.arg_spec if r == "vec_in"},
        "mat_shapes": {n: list(walk.slot_types[("mat_in", n)].shape)
                       for r, n in walk.arg_spec if r == "mat_in"},
        "params": sc._params(walk),
        "accum_outputs": [n for r, n in walk.arg_spec if r == "accum_out"],
        **({"param_planes": list(walk.param_planes)} if walk.param_planes else {}),
        **({"cells": walk.cells} if walk.cells else {}),
        "digest": walk.digest,
    }


def _slot_records(walk) -> list:
    """Per slot, in arg_spec order: role, name, dtype and shape of the plane."""
    out = []
    for role, name in walk.arg_spec:
        t = walk.slot_types[(role, name)]
        out.append({"role": role, "name": name, "dtype": t.dtype,
                    "shape": [int(e) for e in t.shape]})
    return out


#: Registers per thread above which an entry is register-bound: at most one
#: 256-thread block is resident per SM, too few warps for plain loads to keep
#: HBM busy.  Such an entry is rebuilt with two resident blocks asked of the
#: compiler (a 128-register cap); if that build spills, its inputs are staged
#: through shared memory instead.  Measured on the B200 for the SPD-solve VJP
#: (227 registers uncapped): capped to 102 registers without a spill it
#: ran at 83 % of HBM, staged at 73 %, uncapped at 59 %; every kernel with two
#: or more resident blocks lost 5-20 % staged and gained nothing from a cap.
REGISTER_BOUND = 128


#: Registers of one quarter of an SM (a warp scheduler's share of the register
#: file); a thread's registers are allocated in units of 8.
QUARTER_REGISTERS = 16384


def warps_per_quarter(regs: int) -> int:
    """Warps of an entry at ``regs`` registers a thread that one quarter of an
    SM holds (at most 16)."""
    alloc = max(8, -(-regs // 8) * 8)
    return min(16, QUARTER_REGISTERS // (alloc * 32))


def next_slot_bounds(regs: int):
    """``(threads, blocks)`` asking the compiler for one more resident warp per
    quarter of the SM than ``regs`` allows -- 128-thread blocks, four warps a
    block, one block per quarter per warp -- or None at the 16-warp limit.
    Measured on the B200 (full-size configurations): where that cap compiles
    without a spill it is kept, SPD solve 0.67 -> 0.75 and its VJP 0.79 -> 0.85
    of HBM (98 and 102 registers capped to 96: four warps a quarter to five),
    gravity and the energy JVP unchanged; every cap that spilled was slower
    (Kepler, its VJP, the gravity JVP and VJP, the Param-gradient VJP, 2-11 %)."""
    w = warps_per_quarter(regs)
    if w >= 16:
        return None
    return 128, w + 1


def _spills(ptxas: dict, name: str) -> bool:
    r = ptxas.get(name, {})
    return bool(r.get("spill_store_B") or r.get("spill_load_B"))


def build_split_kernel(kernel, directory, *, name: str | None = None, mode: str = "float64") -> dict:
    """A kernel the reference's split cuts into stages (team-form linear
    algebra): one unit holding every stage's entry, one CUBIN, one sidecar
    listing the stages and the scratch planes (target/split.py)."""
    from .split import cell_planes, render_split_unit, user_slots

    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    name = name or kernel.name
    unit, stages, block, members = render_split_unit(kernel, name, mode)
    cubin, _log, ptxas = compile_cubin(unit.text, name)
    stem = f"{name}.{mode}"
    (directory / f"{stem}.cu").write_text(unit.text)
    (directory / f"{stem}.cubin").write_bytes(cubin)
    sidecar = _reference_sidecar(name, members[0].walk, mode, getattr(kernel, "lane_space", None))
    sidecar = json.loads(json.dumps(sidecar, default=str))
    sidecar.update(json.loads(json.dumps(block, default=str)))
    keyed = set(block.get("keyed") or {})
    keyed |= {c for m in members for c, t in (m.walk.companions or {}).items() if t in keyed}
    scratch = set(block.get("team_planes") or {}) | cell_planes(block.get("cells") or {}) | keyed
    sidecar["b200"] = {
        "entry": name,
        "arch": ARCH,
        "unit": f"{stem}.cu",
        "cubin": f"{stem}.cubin",
        "unit_digest": unit.digest,
        "frame": "split",
        "dynamic_smem": 0,
        "stages": 0,
        "min_blocks": 0,
        "persist": None,
        "range": None,
        "step_fp64_ops": None,
        "lane_refill": False,
        "folds": {},
        "sample_sums": [],
        "split": stages,
        "slots": user_slots(stages, scratch),
        "nvrtc_options": [o for o in options() if not o.startswith("-I")],
        "ptxas": ptxas,
    }
    (directory / f"{stem}.json").write_text(json.dumps(sidecar, indent=1, sort_keys=True))
    return sidecar


def choose_unit(kernel, name: str, mode: str = "float64", staged: bool | None = None,
                bounds: tuple | None = None) -> tuple:
    """The unit the b200 row builds for a (not split) kernel and its compile:
    ``(unit, cubin, log, ptxas)``.  The policy, by the entry's registers:
    above ``REGISTER_BOUND`` a cap to two 256-thread blocks a SM, or staged
    inputs where that cap spills; then, one warp slot short of the next, the
    cap ``next_slot_bounds`` gives where it does not spill.  ``staged`` True
    asks for the staged unit, ``bounds`` for a fixed ``(threads, blocks)``."""
    if bounds is not None:
        unit = render_unit(kernel, name, mode, staged=False, threads=bounds[0], min_blocks=bounds[1],
                           warp_tiled=False)
    else:
        unit = render_unit(kernel, name, mode, staged=bool(staged))
    cubin, log, ptxas = compile_cubin(unit.text, name)
    if bounds is None and staged is None and ptxas.get(name, {}).get("regs", 0) > REGISTER_BOUND:
        capped = render_unit(kernel, name, mode, staged=False, min_blocks=2)
        c_cubin, c_log, c_ptxas = compile_cubin(capped.text, name)
        if not _spills(c_ptxas, name):
            unit, cubin, log, ptxas = capped, c_cubin, c_log, c_ptxas
        else:
            trial = render_unit(kernel, name, mode, staged=True)
            if trial.notes.get("staged"):
                unit = trial
                cubin, log, ptxas = compile_cubin(unit.text, name)
    slot = next_slot_bounds(ptxas.get(name, {}).get("regs", 0))
    if (bounds is None and slot is not None and not unit.notes.get("staged") and not unit.notes.get("dynamic_smem")
            and not unit.notes.get("private_smem") and getattr(kernel, "one_step", None) is None):
        capped = render_unit(kernel, name, mode, staged=False, threads=slot[0], min_blocks=slot[1],
                             warp_tiled=False)
        c_cubin, c_log, c_ptxas = compile_cubin(capped.text, name)
        if not _spills(c_ptxas, name):
            unit, cubin, log, ptxas = capped, c_cubin, c_log, c_ptxas
    return unit, cubin, log, ptxas


def b200_block(unit, walk, ptxas: dict, name: str, unit_file: str, cubin_file: str) -> dict:
    """The sidecar's ``b200`` block: what the b200 runtime binds and launches
    from (the entry, its frame, sample sums, slot records, register policy,
    the NVRTC options and the ptxas report)."""
    return {
        "entry": name,
        "arch": ARCH,
        "unit": unit_file,
        "cubin": cubin_file,
        "unit_digest": unit.digest,
        "frame": unit.frame,
        "dynamic_smem": unit.notes.get("dynamic_smem", 0),
        "stages": unit.notes.get("stages", 0),
        "warp_tiled": unit.notes.get("warp_tiled", False),
        "min_blocks": unit.notes.get("min_blocks", 0),
        "block": unit.notes.get("block", 256),
        "persist": unit.notes.get("persist"),
        "range": unit.notes.get("range"),
        "step_fp64_ops": unit.notes.get("step_fp64_ops"),
        "lane_refill": unit.notes.get("lane_refill", False),
        "folds": unit.notes.get("folds") or {},
        "private_targets": unit.notes.get("private_targets") or [],
        "sample_sums": [{"name": n, "op": op, "companion": comp} for n, op, comp in unit.sums],
        "slots": _slot_records(walk),
        "nvrtc_options": [o for o in options() if not o.startswith("-I")],
        "ptxas": ptxas,
    }


def build_kernel(kernel, directory, *, name: str | None = None, mode: str = "float64",
                 staged: bool | None = None, bounds: tuple | None = None) -> dict:
    """Render, compile and write one kernel's b200 artifact; returns its sidecar.
    ``staged`` streams the inputs through TMA-filled shared-memory stages;
    ``None`` decides by the unstaged entry's register count.  A kernel the
    reference's split cuts into stages is built by ``build_split_kernel``."""
    from .split import expand

    name = name or kernel.name
    if expand(kernel, name, mode) is not None:
        return build_split_kernel(kernel, directory, name=name, mode=mode)
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    unit, cubin, log, ptxas = choose_unit(kernel, name, mode, staged, bounds)
    stem = f"{name}.{mode}"
    (directory / f"{stem}.cu").write_text(unit.text)
    (directory / f"{stem}.cubin").write_bytes(cubin)
    sidecar = _reference_sidecar(name, kernel.walk, mode, getattr(kernel, "lane_space", None))
    sidecar = json.loads(json.dumps(sidecar, default=str))
    sidecar["b200"] = b200_block(unit, kernel.walk, ptxas, name, f"{stem}.cu", f"{stem}.cubin")
    (directory / f"{stem}.json").write_text(json.dumps(sidecar, indent=1, sort_keys=True))
    return sidecar


def build(kernels, directory, *, modes=("float64",)) -> dict:
    """Build every kernel in every mode; ``{(name, mode): sidecar}``."""
    out = {}
    for kernel in kernels:
        for mode in modes:
            try:
                out[(kernel.name, mode)] = build_kernel(kernel, directory, mode=mode)
            except HawkError:
                raise
    return out
