"""One b200 translation unit around the reference renderer's body.

The b200 counterpart of the reference's ``render_source``
(hawk/emit/wrapper.py:1132-1271): the body STRING is rendered by the
reference's one renderer (``render_body``, hawk/emit/render.py:140) through the
b200 writer; the unit around it -- prelude, self-check exports, entry
signature, unpack, frame -- is this build's.  The prelude includes the
hand-written sm_100a device library (``hk/hawk_b200.cuh``) instead of the
reference's third-party numerics headers, so the unit compiles under NVRTC with
nothing else on the include path.

Everything the b200 target does not build is refused here, by name, before any
text reaches a compiler.
"""

from __future__ import annotations

import hashlib
import re
from dataclasses import dataclass, field

from ..errors import HawkError
from .persist import RANGE_SUFFIX, SUFFIX as PERSIST_SUFFIX, persist_entry, range_entry, step_fp64_ops
from .refill import refill_frame
from .wrapper import B200, StagePlan, lane_frame_staged, sample_sum_store
from .writer import B200_WRITER, body_text

#: Scalar modes the b200 target builds, each with its C++ element type: the
#: reference's float64, float32 and banded (hawk/emit/wrapper.py:136-143).  A
#: banded value on the b200 target is an IEEE binary64 in its 8-byte cell (this
#: build's own cell format; the reference's packed BandedReal is defined only by
#: the absent aether-dsc): every operation is correctly rounded, within the
#: 0.5 ULP53 a banded op is certified to, and a sum over samples keeps the
#: banded row contract (each row's compensated pair rounded once).
MODES = {"float64": "double", "float32": "float", "banded": "double"}

#: Library namespaces the device library does not provide: a body naming one is
#: refused with the construct it stands for.
_UNBUILT = {
    "hk::rt::": "runtime-index stores and rolled products (aether::rt) other than the rolled store",
    "hk::geometry::": "ray primitives",
    "hk::banded::": "the banded scalar mode",
    "hk::random::": "in-kernel random draws",
    "hawk_abi::mix_count": "auto dispatch branch counts",
    "hawk_abi::tiled": "wide (tiled) scratch planes",
    "hawk_abi::warp_sum": "warp-per-lane sums",
    "hawk_abi::spacing": "the spacing op",
}


#: The entries of the reference's feature table (hawk/targets/features.py:74-152)
#: the b200 row builds; a kernel using any other is refused by the table's own
#: predicate, with its reason and the alternative it names.
BUILT_FEATURES = frozenset({"linalg", "sample_reduction", "cross_sample_at", "compensated", "two_path",
                            "zero_trip_loop"})


def refuse_features(name: str, kernel, walk, sinks) -> None:
    """Refuse the first feature of the reference's table that the kernel uses
    and the b200 row does not build, by name (the reference's C row refuses
    the same way, hawk/embedded/verify.py:110-123)."""
    from hawk.embedded.verify import _every_node, _top
    from hawk.targets import FEATURES

    kind = getattr(kernel, "kind", None)
    nodes = list(_every_node(_top(sinks)))
    for feature, (predicate, (why, fix)) in FEATURES.items():
        if feature in BUILT_FEATURES:
            continue
        hit = predicate(kernel, kind, walk, nodes)
        if hit is not None:
            raise HawkError(f"{name!r}: the b200 target does not build the feature {feature!r} "
                            f"(at {hit[1]} {hit[0]}): {why}; {fix}")


def refuse_banded(name: str, kernel, walk, sinks) -> None:
    """What the banded mode does not build: the ops the reference refuses in
    it (hawk/emit/wrapper.py:179-213: an atomic scattered add, the
    uncertified math functions), any scattered commit (the reference routes a
    banded build's compensated scatter to ordered stages, which this mode does
    not build), and kernels its split cuts into stages."""
    from hawk.emit.wrapper import BANDED, refuse_uncertified

    if walk.companions or any(str(k).startswith("accum") for k in walk.kinds):
        raise HawkError(f"{name!r}: a scattered commit is not built in scalar mode 'banded' on the b200 target "
                        "(a cell has no atomic add, and the ordered stages the reference routes a banded "
                        "scatter to are not built banded here); build this kernel in float64 or float32")
    try:
        refuse_uncertified(sinks, walk, BANDED)
    except Exception as exc:                     # the reference's HawkError, re-raised as this path's
        raise HawkError(f"{name!r}: {exc}") from None
    if getattr(kernel, "team", None) is not None:
        raise HawkError(f"{name!r}: a kernel split into stages is not built in scalar mode 'banded' on the b200 "
                        "target; build it in float64 or float32")


#: The team-form calls the device library builds (hk/team.cuh).
TEAM_BUILT = frozenset({"Team", "TeamCholesky", "TeamLu", "cholesky", "choleskyFrom", "choSolve", "triLower",
                        "triUpperT", "lu", "luSolve", "luSolveT", "luInverse", "luDet", "blockSum",
                        "TeamEigh", "eigh", "TeamQr", "qr", "qrSolve", "qrGramSolve", "scatterChunk",
                        "orderedPart"})
_TEAM_NAME = re.compile(r"hk::linalg::team::(\w+)")


def refuse_unbuilt(name: str, body: str) -> None:
    """Refuse, by the construct it stands for, a body naming what the device
    library does not provide."""
    for token, what in _UNBUILT.items():
        if token == "hk::rt::":
            if re.search(r"hk::rt::(?!store\()", body):
                raise HawkError(f"{name!r}: its body uses {what}, which the b200 target does not build yet")
            continue
        if token in body:
            raise HawkError(f"{name!r}: its body uses {what}, which the b200 target does not build yet")
    for call in sorted(set(_TEAM_NAME.findall(body)) - TEAM_BUILT):
        raise HawkError(f"{name!r}: its team stage calls hk::linalg::team::{call} (team-form "
                        f"{'eigensolver' if 'eigh' in call.lower() else 'QR' if 'qr' in call.lower() else 'block sums' if 'block' in call.lower() else call}), which the b200 target does not build yet")


@dataclass(frozen=True)
class Unit:
    """One emitted unit: its text, the entry name, and the facts the sidecar records."""

    name: str
    mode: str
    text: str
    body: str
    frame: str                      # "lane" or "row"
    sums: tuple = ()                # ((name, op, companion or None), ...) in column order
    digest: str = ""
    notes: dict = field(default_factory=dict)
    entries: str = ""               # the text after the prelude: the entry (and its fold / persist entries)


def prelude_lines(name: str, mode: str, defines=()) -> list:
    """The head of a unit: the build's settings for the device library
    (``defines``), the library, the scalar-mode aliases and the self-check
    exports (hawk/artifact/layout.py:35-61)."""
    return [
        f"// hawk_b200 unit {name!r} (scalar mode {mode}), sm_100a.",
        "// Body text: the reference renderer's; entry, views and frame: the b200 wrapper.",
        *(f"#define {d}" for d in defines),
        '#include "hk/hawk_b200.cuh"',
        "",
        f"using Real = {MODES[mode]};",
        "using Int = long long;",
        "",
        "HK_SELF_CHECK_EXPORTS",
    ]


def _team_prefix() -> str:
    from hawk.ir.team import PLANE_PREFIX
    return PLANE_PREFIX


def _refuse(name: str, walk) -> None:
    for role, slot in walk.arg_spec:
        # a team stage's scratch plane (hawk/ir/team.py PLANE_PREFIX) is the split's; any other wide plane is not built
        if role == "wide_in" or (role == "wide_out" and not slot.startswith(_team_prefix())):
            raise HawkError(f"{name!r}: slot {slot!r} has role {role!r}, which the b200 target does not build")


def _word_read() -> str:
    """The automatic kernel's ``fused_steps`` word, read once per launch."""
    from hawk.emit.spelling import binding_name
    from hawk.ir.nodes import FUSED_STEPS_PLANE

    return f"{binding_name('lookup', FUSED_STEPS_PLANE)}[hk::SampleIndex::make(0)].eval()"


def render_unit(kernel, name: str | None = None, mode: str = "float64", staged: bool = True,
                min_blocks: int | None = None, threads: int | None = None, warp_tiled: bool = True) -> Unit:
    """The b200 unit of a traced kernel (``hawk.Kernel``) in scalar mode ``mode``;
    ``staged`` streams its inputs through shared-memory stages filled by the
    TMA unit (hk/stage.cuh) where the stage plan fits; ``min_blocks`` caps the
    entry's registers so that that many blocks of ``threads`` (256 when None)
    stay resident per SM; ``warp_tiled`` lets a row frame fetch each warp's
    next trip ahead where the wrapper takes it (``B200.warp_tiled``)."""
    from hawk.ir.nodes import sample_sums
    from hawk.emit.render import render_body
    from hawk.emit.spelling import element_spelling

    if mode not in MODES:
        raise HawkError(f"scalar mode {mode!r} is not built on the b200 target (built: {sorted(MODES)})")
    name = name or kernel.name
    walk, sinks = kernel.walk, kernel.sinks
    _refuse(name, walk)
    refuse_features(name, kernel, walk, sinks)
    if mode == "banded":
        refuse_banded(name, kernel, walk, sinks)
    kind = getattr(kernel, "kind", None)
    rendered = render_body(sinks, walk, indent="        ", kind=kind, writer=B200_WRITER)
    body = body_text(rendered.text)
    refuse_unbuilt(name, body)
    sums = sample_sums(sinks)
    if len({s.op for s in sums}) > 1:
        raise HawkError(f"{name!r}: one kernel reduces over samples with one op (sum, max or min)")
    one_step = getattr(kernel, "one_step", None)
    if one_step is not None and sums:
        raise HawkError(f"{name!r}: an automatic stepping kernel with sample sums is not built on the b200 target")
    wrapper = B200
    smem = 0
    frame_note = None
    tiled = False
    elem_bytes = 4 if mode == "float32" else 8
    if sums:
        elem = element_spelling(sums[0].ttype.dtype)
        store = sample_sum_store(sums, banded=mode == "banded")
        plan = StagePlan(walk, elem_bytes, 256 * wrapper.fold_rows(len(sums))) if staged else None
        tile = StagePlan(walk, elem_bytes, 32 * wrapper.fold_rows(len(sums))) if warp_tiled else None
        if plan is not None and plan.enabled:
            opened, closed = wrapper.sample_sum_frame_staged(plan, len(sums), elem, store, sums[0].op,
                                                             elem_bytes=elem_bytes)
            smem = plan.smem_bytes
        elif tile is not None and tile.enabled and wrapper.warp_tiled(tile, len(sums), elem_bytes):
            opened, closed = wrapper.sample_sum_frame_warp_tiled(tile, len(sums), elem, store, sums[0].op,
                                                                 elem_bytes=elem_bytes)
            plan, tiled = tile, True
            smem = 128 + 8 * tile.stage_bytes
        else:
            plan = None
            opened, closed = wrapper.sample_sum_frame(len(sums), elem, store, sums[0].op, elem_bytes=elem_bytes)
        loop = [opened, body, closed]
        frame = "row"
    else:
        plan = StagePlan(walk, elem_bytes, 256) if staged else None
        if plan is not None and plan.enabled:
            opened, closed = lane_frame_staged(plan)
            loop = [opened, body, closed]
            smem = plan.smem_bytes
        else:
            plan = None
            refill = refill_frame(kernel, walk) if one_step is None else None
            loop = [refill] if refill is not None else [wrapper.index_prologue(), body, wrapper.index_epilogue()]
            if refill is not None:
                frame_note = "refill"
        if one_step is not None:
            # an automatic kernel (steps="auto", hawk/trace/steps.py): one uniform
            # branch per launch on the fused_steps word -- 1 runs the single step's
            # body, any other word the fused loop (hawk/emit/wrapper.py:1507-1545)
            plan, smem = None, 0
            single = render_body(one_step.sinks, one_step.walk, indent="        ", kind=kind, writer=B200_WRITER)
            loop = [f"    if ({_word_read()} == 1) {{",
                    wrapper.index_prologue(), body_text(single.text), wrapper.index_epilogue(),
                    "    } else {",
                    wrapper.index_prologue(), body, wrapper.index_epilogue(),
                    "    }"]
        frame = "lane"
    # the run state of each keyed commit target the body names (hk/accum.cuh)
    states = sorted(set(re.findall(r"\bhawk_run_(\w+)\b", "\n".join(loop))))
    run_states = [f"    hk::accum::run::State hawk_run_{t}{{}};" for t in states]
    private = None
    if frame == "lane" and not smem and one_step is None and frame_note is None:
        private = _privatised(walk, body, {x for s in sums for x in (s.name, getattr(s.companion, "name", None))})
    if private is not None:
        head, tail, _targets = private
        loop = [*head, *loop, *tail]
        smem_entry = PRIVATE_BYTES
    else:
        smem_entry = 0
    prelude = [*prelude_lines(name, mode), *([f"HK_DYNAMIC_SMEM({smem})"] if smem else []), ""]
    parts = [
        *([f'extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__{name} = {smem_entry}u;']
          if smem_entry else []),
        wrapper.entry_signature(walk, name, min_blocks, threads),
        "{",
        wrapper.unpack(walk, plan),
        *run_states,
        *loop,
        "}",
        "",
    ]
    folds = {}
    for comp, target in (walk.companions or {}).items():
        # the owned companion's fold: one lane per slot of the target, launched
        # after the kernel (hawk/emit/wrapper.py:1274-1293)
        from hawk.emit.spelling import binding_name

        fold = f"{name}__fold_{target}"
        folds[target] = fold
        parts += [wrapper.entry_signature(walk, fold), "{", wrapper.unpack(walk, None), wrapper.index_prologue(),
                  f"        hawk_abi::fold_companion({binding_name('accum_out', target)}, "
                  f"{binding_name('accum_out', comp)}, i);",
                  wrapper.index_epilogue(), "}", ""]
    persist = persist_entry(kernel, name, wrapper) if one_step is not None else None
    if persist is not None:
        parts += [persist, ""]
    ranged = range_entry(kernel, name, wrapper) if one_step is not None else None
    if ranged is not None:
        parts += [ranged, ""]
    entries = "\n".join(parts)
    text = "\n".join(prelude) + "\n" + entries
    records = tuple((s.name, s.op, s.companion.name if s.op == "sum" else None) for s in sums)
    return Unit(name=name, mode=mode, text=text, body=body, frame=frame, sums=records, entries=entries,
                digest=hashlib.sha256(text.encode()).hexdigest(),
                notes={"dynamic_smem": smem, "staged": plan is not None and not tiled,
                       "stages": plan.stages if plan is not None and not tiled else 0, "warp_tiled": tiled,
                       "min_blocks": min_blocks or 0,
                       "block": threads or 256,
                       "persist": f"{name}{PERSIST_SUFFIX}" if persist is not None else None,
                       "range": f"{name}{RANGE_SUFFIX}" if ranged is not None else None,
                       "step_fp64_ops": step_fp64_ops(kernel) if persist is not None else None,
                       "lane_refill": frame_note == "refill", "folds": folds,
                       "private_targets": [t for t, _k, _c in (private[2] if private else ())],
                       "private_smem": smem_entry})


_IDENT = re.compile(r"[A-Za-z_][A-Za-z0-9_]*")

#: Dynamic shared memory of an entry that privatises its scatter targets: per
#: block, the targets' copies (a target whose plane does not fit its share
#: commits to the plane).  At 32 KB, seven 256-thread blocks stay resident.
PRIVATE_BYTES = 32 * 1024

_COMMITS = (
    (re.compile(r"hawk_abi::accum_add_compensated\((\w+), (\w+),"), "compensated"),
    (re.compile(r"hk::accum::run::add(?:Tested|Sorted)?Compensated(?:<\d+>)?\((\w+), (\w+),"), "compensated"),
    (re.compile(r"hawk_abi::accum_add\((\w+),"), "add"),
    (re.compile(r"hk::accum::run::add(?:Tested|Sorted)?(?:<\d+>)?\((\w+),"), "add"),
    (re.compile(r"hawk_abi::accum_or\((\w+),"), "or"),
)


def _privatised(walk, body: str, row_planes: set):
    """``(head, tail, targets)`` of an entry whose scattered commits go through
    block-private copies of their targets (hk::accum::privatise), or None.
    A target the body commits one way only (plain, compensated with its
    companion, or OR) is privatised; the copies shadow the targets' views for
    the loop, and the block adds them into the planes when it leaves."""
    from hawk.emit.spelling import binding_name

    scatter = {binding_name(role, name) for role, name in walk.arg_spec
               if role == "accum_out" and name not in row_planes}
    if re.search(r"hk::accum::run::add(?:Compensated)?<\d+>\(", body):
        return None     # aligned runs already commit once per run of lanes: a copy gains little
    kinds: dict = {}
    comps: dict = {}
    for pattern, kind in _COMMITS:
        for m in pattern.finditer(body):
            target = m.group(1)
            if target not in scatter:
                return None
            kinds.setdefault(target, set()).add(kind)
            if kind == "compensated":
                comps.setdefault(target, set()).add(m.group(2))
    if not kinds:
        return None
    targets = []
    for target, ks in sorted(kinds.items()):
        if len(ks) != 1 or (ks == {"compensated"} and len(comps[target]) != 1):
            return None
        kind = next(iter(ks))
        targets.append((target, kind, next(iter(comps[target])) if kind == "compensated" else None))
    named = [t for t, _k, _c in targets] + [c for _t, _k, c in targets if c]
    head = ["    hk::accum::PrivSpace hawk_ps = hk::accum::private_space();"]
    head += [f"    const auto hawk_pv_{b} = hk::accum::privatise(hawk_ps, {b});" for b in named]
    head += ["    __syncthreads();", "    {"]
    head += [f"    const auto& {b} = hawk_pv_{b};" for b in named]
    tail = ["    }", "    __syncthreads();"]
    for target, kind, comp in targets:
        if kind == "compensated":
            tail.append(f"    hk::accum::flush_compensated(hawk_pv_{target}, hawk_pv_{comp});")
        elif kind == "or":
            tail.append(f"    hk::accum::flush_or(hawk_pv_{target});")
        else:
            tail.append(f"    hk::accum::flush_add(hawk_pv_{target});")
    return head, tail, targets
