"""Split kernels on the b200 target: every stage of a kernel in one unit.

A kernel whose team-form linear algebra (a matrix above the one-thread cap,
hawk/ir/team.py) cannot run in one launch is cut by the reference's own split
(``_expand_split``, hawk/artifact/bundle.py:1177-1275; hawk/ir/split.py:304)
into stages named ``<name>``, ``<name>_2``, ...:

* a copy stage (a plain kernel with a team): the lane's operands stored
  row-major into runtime-owned scratch planes (``tm*``), one block per lane;
* a team stage (``TeamStage``): the reference's team body
  (hawk/emit/team.py:466), collective calls into ``hk::linalg::team``;
* a reader stage: a plain per-lane kernel that reads the results back.

The reference builds each stage as an artifact of its own and its runtime
launches them in order over scratch it allocates (hawk/runtime.py:675-748).
Here the stages are the entries of ONE unit (one CUBIN, one sidecar): a team
entry exports its block size (``hk_team_threads__<entry>``) and the dynamic
shared memory its calls stage into (``hk_dynamic_smem_bytes__<entry>``), which
the loader reads; the sidecar lists the stages, their slots and the scratch
planes (``team_planes``) for the runtime's split runner.
"""

from __future__ import annotations

import hashlib
import re

from ..errors import HawkError
from .assemble import MODES, Unit, prelude_lines, refuse_unbuilt, render_unit
from .wrapper import B200
from .writer import B200_WRITER, body_text

#: Dynamic shared memory the teams of one SM may stage into (of its 228 KB).
TEAM_SMEM_LIMIT = 220 * 1024
#: Teams (warps, one lane each) per SM that must fit staged for a stage to
#: stage at all: below it, working in place through L1/L2 with more lanes in
#: flight is the faster of the two.
TEAM_STAGED_WARPS = 6
#: Warps per block of a team entry that works in place (a staged one takes one
#: warp per block, so as many blocks as fit share an SM).
TEAM_WARPS_IN_PLACE = 4


def _round16(b: int) -> int:
    return (b + 15) & ~15


def _inplace_bytes(n: int, elem: int) -> int:
    """hk::linalg::team::inplace_bytes: the head (the staged-factor tag) and
    the products row of the backward sweeps."""
    return 128 + _round16(elem * n)


def _staged_bytes(n: int, k: int, elem: int) -> int:
    """hk::linalg::team::staged_bytes: the in-place part, the matrix (row
    stride n + 1), the right-hand sides."""
    return _inplace_bytes(n, elem) + _round16(elem * n * (n + 1)) + _round16(elem * n * k)


#: Team calls that read and write only a factor's lower triangle; staged, it
#: is packed (hk::linalg::team::staged_lower_bytes).
LOWER_OPS = frozenset({"chol", "chol_from", "cho_solve", "tri_lower", "tri_upper_t"})


def _staged_lower_bytes(n: int, k: int, elem: int) -> int:
    """hk::linalg::team::staged_lower_bytes: the in-place part, the packed
    lower triangle, the right-hand sides."""
    return _inplace_bytes(n, elem) + _round16(elem * n * (n + 1) // 2) + _round16(elem * n * k)


def team_geometry(spec, elem: int) -> tuple:
    """``(threads, smem)`` of a team stage's block.  A team is one warp
    (hk/team.cuh).  When the largest staged need of the stage's calls leaves
    room for TEAM_STAGED_WARPS teams per SM, a block is one team with that much
    dynamic shared memory; else a block is TEAM_WARPS_IN_PLACE teams with none
    (the calls work in place on the scratch planes, through L1 and L2)."""
    needs, inplace = [], [0]
    for step in spec.steps:
        n = int(step.n)
        k = n if step.op == "lu_inverse" else int(step.k or 0)
        needs.append(_staged_lower_bytes(n, k, elem) if step.op in LOWER_OPS else _staged_bytes(n, k, elem))
        inplace.append(_inplace_bytes(n, elem))
    if needs and max(needs) * TEAM_STAGED_WARPS <= TEAM_SMEM_LIMIT:
        return 32, max(needs)
    return 32 * TEAM_WARPS_IN_PLACE, max(inplace) * TEAM_WARPS_IN_PLACE


def lower_staged(spec, smem: int, threads: int) -> bool | None:
    """Whether the Cholesky-family calls of a team stage stage their packed
    triangle (True), work in place (False), or the stage makes none (None)."""
    lower = [st for st in spec.steps if st.op in LOWER_OPS]
    if not lower:
        return None
    return threads == 32 and smem > 0


def expand(kernel, name: str, mode: str = "float64"):
    """``(members, block)``: the stage kernels and the reference's sidecar block
    (stages, cells, team_planes), or None for a kernel that runs in one launch.

    A kernel that runs in one launch under the reference's general split may
    still have a warp entry on a device-only sm_100 build (an eigenvalues-only
    32 x 32 eigh, hawk/ir/team.py:236-275): then it is cut the way the
    reference cuts it there, into a copy, an ``eigh_warp`` and a reader
    stage."""
    from hawk.artifact.bundle import _expand_split
    from hawk.emit import policy
    from hawk.targets.cards import _BUILD_ARCH
    from hawk.trace.kernel import TeamStage

    members, names, _kinds, blocks = _expand_split([kernel], [name], [None], device=True, device_only=False)
    block = blocks.get(name)
    if block is not None and len(members) >= 2:
        return members, block
    token = _BUILD_ARCH.set("sm_100")
    try:
        with policy.using(scalar=mode, device_only=True):
            members, names, _kinds, blocks = _expand_split([kernel], [name], [None], device=True, device_only=True)
    finally:
        _BUILD_ARCH.reset(token)
    block = blocks.get(name)
    warp = any(isinstance(mm, TeamStage) and any(st.op == "eigh_warp" for st in mm.team.steps) for mm in members)
    if block is None or len(members) < 2 or not warp:
        return None
    return members, block


def _threads(member) -> int | None:
    team = getattr(member, "team", None)
    if team is None:
        return None
    t = int(team.threads)
    if t % 32 or t <= 0 or t > 1024:
        raise HawkError(f"{member.name!r}: a team of {t} threads is not whole warps (1 to 32 of them)")
    return t


def render_split_unit(kernel, name: str, mode: str = "float64"):
    """``(unit, stages, block)``: the unit holding every stage's entry, the
    per-stage records and the reference's split block."""
    from hawk.trace.kernel import TeamStage

    if mode not in MODES:
        raise HawkError(f"scalar mode {mode!r} is not built on the b200 target (built: {sorted(MODES)})")
    found = expand(kernel, name, mode)
    if found is None:
        raise HawkError(f"{name!r} runs in one launch; it is not a split kernel")
    members, block = found
    elem = 4 if mode == "float32" else 8
    parts, stages = [], []
    lower_modes: set = set()
    for member, record in zip(members, block["stages"]):
        if getattr(member, "one_step", None) is not None:
            raise HawkError(f"{name!r}: an automatic stepping kernel's stages are not built on the b200 target")
        threads = _threads(member)
        walk = member.walk
        if threads is None:
            # a per-lane stage: the lane frame, or the row frame of the sample
            # sums it reduces into cells a later stage reads
            unit = render_unit(member, member.name, mode, staged=False, warp_tiled=False)
            if unit.notes.get("persist") or unit.notes.get("folds"):
                raise HawkError(f"{name!r}: stage {member.name!r} commits into a compensated scatter target, "
                                "which a split kernel's stage does not build yet")
            copies = _reader_copies(unit, walk) if not unit.sums else None
            if copies is not None:
                parts += _reader_entry(member.name, walk, copies)
                stages.append({"entry": member.name, "kind": "team", "threads": READER_THREADS, "dynamic_smem": 0,
                               "slots": _slot_records(walk), "sample_sums": [],
                               "cells_in": list(record.get("cells_in") or ()), "cells_out": [], "grid": "lanes",
                               "keyed": None, "groups": None, "of": None, "status": None, "ops": ["copy_out"]})
                continue
            parts.append(unit.entries)
            stages.append({"entry": member.name, "kind": unit.frame, "threads": None, "dynamic_smem": 0,
                           "slots": _slot_records(walk), "lane_refill": unit.notes.get("lane_refill", False),
                           "sample_sums": [{"name": n, "op": op, "companion": comp} for n, op, comp in unit.sums],
                           "cells_in": list(record.get("cells_in") or ()),
                           "cells_out": list(record.get("cells_out") or ())})
            continue
        if record.get("cells_in") or record.get("cells_out"):
            raise HawkError(f"{name!r}: team stage {member.name!r} reads or makes a sample sum, which the b200 "
                            "target does not build yet")
        if isinstance(member, TeamStage):
            body = body_text(member.fused_body().text)
            threads, smem = team_geometry(member.team, elem)
            if "__shared__" in body:
                # the body keeps arrays of its own in shared memory: one team a block
                threads, smem = 32, (smem // max(threads // 32, 1) if smem else 0)
            staged_lower = lower_staged(member.team, smem, threads)
            if staged_lower is not None:
                lower_modes.add(staged_lower)
            if "hawk_map" in body:
                raise HawkError(f"{name!r}: a block sum over an index map (an active-set build) is not built "
                                "on the b200 target")
            for step in member.team.steps:
                if step.op == "block_part":
                    body = _ordered_part(body)
            chunked = [st for st in member.team.steps if st.op == "scatter_chunks"]
            if chunked:
                if len(member.team.steps) != 1:
                    raise HawkError(f"{name!r}: stage {member.name!r} walks an ordered scatter's chunks beside "
                                    "other steps, which the b200 target does not build")
                body, threads = _scatter_chunk_body(chunked[0]), 32     # the bins are the block's
        else:                       # a copy stage: the stage's own sinks, a block per lane
            from hawk.emit.render import render_body

            body = body_text(render_body(member.sinks, walk, indent="        ", kind=getattr(member, "kind", None),
                                         writer=B200_WRITER).text)
            smem = 0
        refuse_unbuilt(member.name, body)
        team_record = dict(record.get("team") or {})
        if isinstance(member, TeamStage) and any(st.op == "scatter_chunks" for st in member.team.steps):
            team_record["groups"] = SCATTER_WARPS       # teams a chunk (hk::linalg::team::scatterChunk)
        spans = team_record.get("grid", "lanes") != "lanes"
        parts += [
            f'extern "C" __device__ const unsigned int hk_team_threads__{member.name} = {threads}u;',
            *([f'extern "C" __device__ const unsigned int hk_team_spans_run__{member.name} = 1u;'] if spans else []),
            f'extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__{member.name} = {smem}u;',
            B200.entry_signature(walk, member.name, threads=threads),
            "{",
            B200.unpack(walk),
            B200.team_prologue(),
            body,
            B200.team_epilogue(),
            "}",
            "",
        ]
        stages.append({"entry": member.name, "kind": "team", "threads": threads, "dynamic_smem": smem,
                       "slots": _slot_records(walk), "sample_sums": [], "cells_in": [], "cells_out": [],
                       "grid": team_record.get("grid", "lanes"), "keyed": team_record.get("keyed"),
                       "groups": team_record.get("groups"), "of": team_record.get("of"),
                       "status": team_record.get("status"),
                       "ops": [st.op for st in member.team.steps] if isinstance(member, TeamStage) else []})
    # every Cholesky-family call of the unit stages its packed triangle, or
    # none does: the library compiles that one accessor (hk/team.cuh)
    defines = [f"HK_TEAM_LOWER_STAGED {int(lower_modes.pop())}"] if len(lower_modes) == 1 else []
    text = "\n".join([*prelude_lines(name, mode, defines), "", *parts])
    unit = Unit(name=name, mode=mode, text=text, body="", frame="split",
                digest=hashlib.sha256(text.encode()).hexdigest(), entries="\n".join(parts),
                notes={"dynamic_smem": 0, "staged": False, "stages": 0, "min_blocks": 0, "persist": None,
                       "step_fp64_ops": None, "lane_refill": False, "folds": {}})
    return unit, stages, block, members


def _ordered_part(body: str) -> str:
    """A plain ordered sum's first stage with its device fill and tree (the
    reference's 1024 virtual lanes a group, hawk/emit/team.py:208-240)
    replaced by ``hk::linalg::team::orderedPart``, which folds only the slots
    that can hold rows: the same bits.  A product of two planes' rows keeps
    the reference's form."""
    lines = body.split("\n")
    fill = next((i for i, ln in enumerate(lines) if ln.strip().startswith(
        "for (std::size_t hawk_t = static_cast<std::size_t>(hawk_tm.rank); hawk_t < 1024;")), None)
    if fill is None or lines[fill - 1].strip() != "#if defined(__CUDA_ARCH__)" \
            or lines[fill + 3].strip() != "hawk_s += hawk_u[hawk_r];":
        return body
    host = next(i for i in range(fill, len(lines)) if lines[i].strip() == "#else")
    endif = next(i for i in range(host, len(lines)) if lines[i].strip() == "#endif")
    tree = next(i for i in range(endif, len(lines))
                if lines[i].strip() == "for (std::size_t hawk_w = 512; hawk_w > 0; hawk_w >>= 1) {")
    if lines[endif + 1].strip() != "hawk_tm.sync();" or lines[tree + 4].strip() != "}":
        return body
    indent = lines[fill - 1][:len(lines[fill - 1]) - len(lines[fill - 1].lstrip())]
    device = [lines[fill - 1],
              f"{indent}hk::linalg::team::orderedPart<Real>(hawk_tm, hawk_u, hawk_rows, hawk_grp, hawk_sh);",
              lines[host], *lines[host + 1:endif], lines[endif + 1], *lines[tree:tree + 5], lines[endif]]
    return "\n".join(lines[:fill - 1] + device + lines[tree + 5:])


#: Warps a lane chunk of an ordered scatter is walked by (each owns the keys
#: of one residue mod this): the reference fixes the chunks at up to 256, so
#: one warp a chunk leaves most of the GPU idle.  2^24 lanes into 1000 cells:
#: 8 warps 0.997 ms, 16 warps 0.928, 32 warps 1.506 (each warp reads the
#: whole chunk's keys).
SCATTER_WARPS = 16


def _scatter_chunk_body(step) -> str:
    """The ordered scatter's chunk stage (the reference's text,
    hawk/emit/team.py:340-436, walks a chunk on one warp with 32 broadcasts
    a batch) as ``hk::linalg::team::scatterChunk``: SCATTER_WARPS warps a
    chunk, each owning the keys of one residue, one match a batch -- each
    partial sum the same operations in the same order, so the same bits."""
    from hawk.emit.spelling import binding_name

    planes = dict(step.planes)
    k, v, part, status = (binding_name("wide_out", planes[r]) for r in ("k", "v", "part", "status"))
    return "\n".join([
        "        const hk::linalg::team::Team hawk_tm = hk::linalg::team::Team::here();",
        "        const long long hawk_lane = hawk_i;",
        f"        {{  // scatter_chunks, n = {int(step.n)}: {SCATTER_WARPS} warps a chunk",
        f"            hk::linalg::team::scatterChunk<Real, {SCATTER_WARPS}>(hawk_tm, hawk_lane, count, nSamples, "
        f"{int(step.n)}, {k}.data(), {v}.data(), {part}.data(), const_cast<std::int32_t*>({status}.data()));",
        "        }"])


#: Threads a block of a reader stage copies its tiles with.
READER_THREADS = 256

_SLICE = re.compile(r"^const hk::Slice<Real, (\d+)(?:, (\d+))?> (hawk_la\d+)\{(\w+)\.data\(\) \+ "
                    r"static_cast<std::size_t>\(static_cast<Int>\(hawk_i\)\) \* (\d+)\};$")
_ALIAS = re.compile(r"^const auto (t\d+) = (hawk_la\d+);$")
_STORE = re.compile(r"^(\w+)\[i\] = (t\d+);$")
_SCALAR = re.compile(r"^(\w+)\[i\] = (\w+)\[hk::SampleIndex::make\(static_cast<std::size_t>\("
                     r"static_cast<Int>\(hawk_i\)\)\)\]\.eval\(\);$")


def _reader_copies(unit, walk) -> list | None:
    """A per-lane stage that only copies team scratch into the kernel's outputs
    (each output the lane's slice of a lane-major scratch plane, or one
    element of it): ``[(output binding, scratch binding, components), ...]``,
    else None.  The reference emits such a stage after a team stage (its
    readers, hawk/emit/team.py): one thread a lane, each copying its lane's
    whole slice -- for a 128 x 128 factor 16384 elements a thread, and only as
    many threads as lanes."""
    from hawk.emit.spelling import binding_name

    comps = {}
    for role, name in walk.arg_spec:
        n = 1
        for e in walk.slot_types[(role, name)].shape:
            n *= int(e)
        comps[binding_name(role, name)] = (role, n)
    slices, temps, out = {}, {}, []
    for raw in unit.body.split("\n"):
        line = raw.strip()
        if not line:
            continue
        m = _SLICE.match(line)
        if m:
            rows, cols, la, src, size = m.groups()
            if int(rows) * int(cols or 1) != int(size):
                return None
            slices[la] = (src, int(size))
            continue
        m = _ALIAS.match(line)
        if m and m.group(2) in slices:
            temps[m.group(1)] = slices[m.group(2)]
            continue
        m = _STORE.match(line)
        if m and m.group(2) in temps:
            src, size = temps[m.group(2)]
            if comps.get(m.group(1), (None, 0))[1] != size:
                return None
            out.append((m.group(1), src, size))
            continue
        m = _SCALAR.match(line)
        if m and comps.get(m.group(1), (None, 0))[1] == 1 and m.group(2) in comps:
            out.append((m.group(1), m.group(2), 1))
            continue
        return None
    return out or None


def _reader_entry(name: str, walk, copies: list) -> list:
    """The reader stage as a team-geometry entry: every block copies 32 x 32
    tiles (``hk::linalg::team::copyOutTile``) of every (output, scratch) pair,
    grid-striding over all pairs' tiles, so the copy runs with 8 warps a 256
    lanes' worth of blocks and reads and writes 32 consecutive elements a warp
    instruction.  Each element is copied unchanged, so the outputs are those
    of the reference's per-lane copy."""
    bounds = []
    lines = ["    __shared__ __align__(16) unsigned char hk_tile[32 * 33 * 8];",
             "    const long long hk_lane_tiles = (count + 31) / 32;"]
    for j, (_dst, _src, size) in enumerate(copies):
        prev = f"hk_end{j - 1} + " if j else ""
        lines.append(f"    const long long hk_end{j} = {prev}hk_lane_tiles * {-(-size // 32)};")
        bounds.append(f"hk_end{j}")
    lines.append(f"    for (long long hk_t = blockIdx.x; hk_t < {bounds[-1]}; hk_t += gridDim.x) {{")
    for j, (dst, src, size) in enumerate(copies):
        pitch = f"{dst}.pitch" if size > 1 else "0ull"
        start = f"hk_t - hk_end{j - 1}" if j else "hk_t"
        cond = f"if (hk_t < hk_end{j})" if j == 0 else (f"else if (hk_t < hk_end{j})" if j < len(copies) - 1
                                                          else "else")
        lines.append(f"        {cond} hk::linalg::team::copyOutTile({src}.data(), {dst}.data(), {pitch}, {size}LL, "
                     f"base, count, {start}, hk_tile);")
    lines += ["    }", "    (void)nSamples;"]
    return [
        f'extern "C" __device__ const unsigned int hk_team_threads__{name} = {READER_THREADS}u;',
        f'extern "C" __device__ const unsigned int hk_dynamic_smem_bytes__{name} = 0u;',
        B200.entry_signature(walk, name, threads=READER_THREADS),
        "{",
        B200.unpack(walk),
        *lines,
        "}",
        "",
    ]


def _slot_records(walk) -> list:
    out = []
    for role, name in walk.arg_spec:
        t = walk.slot_types[(role, name)]
        out.append({"role": role, "name": name, "dtype": t.dtype, "shape": [int(e) for e in t.shape]})
    return out


def cell_planes(cells: dict) -> set:
    """Every plane name a cell stands for between stages: its row planes and
    their companions (hawk/_cells.py:34-36) and the one-cell lookup planes a
    later stage reads (the same names)."""
    out = set()
    for cell, spec in cells.items():
        cols = int(spec.get("columns", 1))
        names = (cell,) if cols == 1 else tuple(f"{cell}_{k}" for k in range(cols))
        out.update(names)
        out.update(f"{n}_comp" for n in names)
    return out


def user_slots(stages: list, scratch) -> list:
    """The slots a caller binds: every stage's, less the runtime's scratch
    planes and the planes of cells (``scratch``), each once (its first
    stage's record).  A cell the caller stores is bound by its own name."""
    seen, out = set(), []
    for st in stages:
        for slot in st["slots"]:
            if slot["name"] in scratch:
                continue
            if slot["name"] in seen:
                continue
            seen.add(slot["name"])
            out.append(slot)
    return out
