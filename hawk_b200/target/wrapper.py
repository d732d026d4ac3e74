"""The b200 Wrapper: how a traced kernel is wrapped for the sm_100a execution model.

It implements the reference's Wrapper protocol (hawk/emit/wrapper.py:225-285;
``qualifier``, ``entry_signature``, ``index_prologue``, ``index_epilogue``,
``unpack``, ``fold_rows``, ``sample_sum_frame``, ``dispatch``) so the reference's
one body renderer (hawk/emit/render.py:140) renders the body unchanged.  What
differs from the reference's CUDA wrapper (hawk/emit/cuda.py:37-794):

* the entry's role arguments are the same by-value mirrors in the same order
  followed by the int64 partition triple (hawk/emit/cuda.py:46-54), but typed by
  this build's own PODs (``hk::abi::*``, equal sizes and field order);
* views are rebuilt as ``hk::`` views over the component-major planes
  (read-only path for inputs, streaming stores for outputs);
* the index seam is a grid-stride loop (the grid is sized by the runtime to
  the SM count times the resident blocks), not one thread per sample;
* a kernel with sample sums runs the row frame: one warp per 32-sample row,
  the row reduced by a register butterfly (hk/sample_sum.cuh) and stored by
  lane ``k`` for column ``k``.

This module imports the reference's front end; it is used where hawk is
importable (to build bundles), never by the runtime.
"""

from __future__ import annotations

from ..errors import HawkError

#: Threads per block every b200 entry is compiled for (``__launch_bounds__``).
BLOCK = 256

#: The roles this wrapper builds, by the view it unpacks them into.
_INPUT_ROLES = ("vec_in", "mat_in", "per_sample", "lookup")
_SINK_ROLES = ("mutable", "out", "accum_out", "wide_out")
_VALUE_ROLES = ("uniform", "nsamples")

_OP_CODE = {"sum": "hk::ss::kSum", "max": "hk::ss::kMax", "min": "hk::ss::kMin"}


def _spelling():
    from hawk.emit import spelling
    return spelling


def param_type(role: str, ttype) -> str:
    """The by-value type one slot crosses the launch as (the reference's
    ``_param_type``, hawk/emit/cuda.py:787-794, with this build's PODs)."""
    sp = _spelling()
    shape = sp.mirror_of(role, ttype)
    if shape == "value":
        if role == "nsamples":
            return "hk::abi::index_t"
        return "Int" if ttype.dtype in sp.INT_PLANE_DTYPES else sp.element_spelling(ttype.dtype)
    return f"hk::abi::{shape}"


def view_decl(role: str, name: str, ttype, stage=None) -> list:
    """The unpack lines of one slot: its view (or by-value local).  ``stage`` is
    ``(offset, component bytes)`` of a staged input in its CTA's stage."""
    sp = _spelling()
    ident = sp.binding_name(role, name)
    src = sp.param_name(role, name)
    elem = sp.element_spelling(ttype.dtype)
    shape = tuple(int(e) for e in ttype.shape)
    if role in _VALUE_ROLES:
        return [f"    const {param_type(role, ttype)} {ident} = {src};", f"    (void){ident};"]
    if role == "terminated":
        # the mask is read through one binding and set through its writable
        # twin (hawk/emit/spelling.py:171-173); both are the same plane
        twin = sp.finish_binding(name)
        return [f"    const hk::MaskView {ident}({src});", f"    (void){ident};",
                f"    const hk::MaskView {twin}({src});", f"    (void){twin};"]
    if role in _INPUT_ROLES:
        if len(shape) == 0:
            view = f"hk::ScalarIn<{elem}>"
        elif len(shape) == 1:
            view = f"hk::VecIn<{elem}, {shape[0]}>"
        elif len(shape) == 2:
            view = f"hk::MatIn<{elem}, {shape[0]}, {shape[1]}>"
        else:
            raise HawkError(f"slot {name!r}: a rank-{len(shape)} input plane is not built on the b200 target")
        args = src
        if stage is not None:
            args += f", {stage[0]}u" + (f", {stage[1]}u" if shape else "")
        return [f"    const {view} {ident}({args});", f"    (void){ident};"]
    if role in _SINK_ROLES:
        if len(shape) == 0:
            view = f"hk::ScalarOut<{elem}>"
        elif len(shape) == 1:
            view = f"hk::VecOut<{elem}, {shape[0]}>"
        elif len(shape) == 2:
            view = f"hk::MatOut<{elem}, {shape[0]}, {shape[1]}>"
        else:
            raise HawkError(f"slot {name!r}: a rank-{len(shape)} sink plane is not built on the b200 target")
        return [f"    const {view} {ident}({src});", f"    (void){ident};"]
    raise HawkError(
        f"slot {name!r} has role {role!r}, which the b200 target does not build "
        f"(built roles: {sorted(_INPUT_ROLES + _SINK_ROLES + _VALUE_ROLES)})")


class B200Wrapper:
    """The b200 half of the wrapper seam."""

    qualifier = "__device__ __forceinline__"

    def entry_signature(self, walk, name: str, min_blocks: int | None = None, threads: int | None = None) -> str:
        """``extern "C" __global__`` entry: role mirrors by value in ``arg_spec``
        order, then the int64 partition triple.  ``min_blocks`` asks the
        compiler to keep that many blocks resident per SM (a register cap);
        ``threads`` is a team entry's block (one team per lane)."""
        sp = _spelling()
        params = [f"    {param_type(role, walk.slot_types[(role, n)])} {sp.param_name(role, n)}"
                  for role, n in walk.arg_spec]
        params += ["    long long base", "    long long count", "    long long nSamples"]
        bounds = f"{threads or BLOCK}, {min_blocks}" if min_blocks else f"{threads or BLOCK}"
        return (f'extern "C" __global__ void __launch_bounds__({bounds}) {name}(\n'
                + ",\n".join(params) + ")")

    def index_prologue(self, segment=None, *, active=None, box=None, team=None) -> str:
        """The lane frame: a grid-stride loop binding ``hawk_i`` and ``i``;
        with ``team`` (the team's threads) the team frame."""
        for label, value in (("segmented", segment), ("active-set", active), ("thread-box", box)):
            if value is not None:
                raise HawkError(f"the {label} entry is not built on the b200 target")
        if team is not None:
            return self.team_prologue()
        return ("    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; "
                "hawk_flat += hk::lane_step()) {\n"
                "        const long long hawk_i = base + hawk_flat;\n"
                "        const hk::SampleIndex i{hawk_i};\n"
                "        (void)hawk_i;\n"
                "        (void)nSamples;")

    def index_epilogue(self) -> str:
        return "    }"

    def team_prologue(self) -> str:
        """The team frame.  The reference makes the lane the block
        (hawk/emit/cuda.py:82-92); here the team of a lane is one warp
        (hk/team.cuh), so a block of the entry's threads serves one lane per
        warp: a grid-stride loop over the partition's lanes by warps, every
        thread of a warp on the same lane (the team's calls are collective);
        the grid is the runtime's, at most the resident blocks."""
        return ("    hk::linalg::team::begin_entry();\n"
                "    const long long hawk_teams = static_cast<long long>(blockDim.x >> 5);\n"
                "    for (long long hawk_flat = static_cast<long long>(blockIdx.x) * hawk_teams + (threadIdx.x >> 5); "
                "hawk_flat < count; hawk_flat += static_cast<long long>(gridDim.x) * hawk_teams) {\n"
                "        const long long hawk_i = base + hawk_flat;\n"
                "        const hk::SampleIndex i{hawk_i};\n"
                "        const Int hawk_wl = static_cast<Int>(threadIdx.x & 31);\n"
                "        (void)hawk_i;\n"
                "        (void)hawk_wl;\n"
                "        (void)nSamples;")

    def team_epilogue(self) -> str:
        """The end of a team trip: the warp leaves the lane together (its part
        of the shared memory is its next lane's)."""
        return "        __syncwarp();\n    }"

    def unpack(self, walk, plan: "StagePlan | None" = None) -> str:
        """Every slot's view, in ``arg_spec`` order; a promoted Param's one-cell
        plane is read once, ahead of the loop (hawk/emit/wrapper.py:1599-1605).
        With a stage plan, each staged input knows its place in the stage."""
        sp = _spelling()
        lines = []
        for role, name in walk.arg_spec:
            ttype = walk.slot_types[(role, name)]
            stage = plan.offsets.get((role, name)) if plan is not None and plan.enabled else None
            lines += view_decl(role, name, ttype, stage)
            if role == "lookup" and name in walk.param_planes:
                cell = sp.param_cell_binding(name)
                lines += [f"    const auto {cell} = {sp.binding_name(role, name)}.cell();",
                          f"    (void){cell};"]
        return "\n".join(lines)

    def fold_rows(self, width: int) -> int:
        """Rows one warp folds per trip: the largest power of two K with
        K * width <= 32 butterfly columns (hk::ss::rows_reduce).  Measured on
        the B200 for the 3-column Param-gradient VJP at 2^26 samples: K = 4,
        8, 16 take 0.429, 0.283, 0.399 ms; a shared-memory variant in which
        each lane evaluates one whole (row, column) tree took 0.375 ms, and
        lane-permuted rows (select-free row rounds, 8 rows per load) 0.387 ms."""
        k = 1
        while k < 32 and 2 * k * width <= 32:
            k *= 2
        return k

    @staticmethod
    def row_lanes(k: int, elem_bytes: int) -> int:
        """Lanes over which each row of a K-row trip is spread (``P`` = 32 / K),
        or 0 for the plain mapping.  Spread, lane l holds samples (l % P) + P q
        of row l / P and the row tree's levels 16 ... P apart are joined in
        registers (hk::ss::rows_reduce_lanes); P lanes read P consecutive
        samples of a row, so the spread is taken only where that is a whole
        32-byte sector (P * element size >= 32)."""
        p = 32 // k
        return p if p * elem_bytes >= 32 and p < 32 else 0

    @staticmethod
    def _flat(lanes: int) -> str:
        """The sample of the trip's slot ``hawk_q`` on this lane, counted from
        the partition's start."""
        if not lanes:
            return "((hawk_r0 + hawk_q) << 5) + static_cast<long long>(threadIdx.x & 31u)"
        shift = lanes.bit_length() - 1
        return (f"((hawk_r0 + static_cast<long long>((threadIdx.x & 31u) >> {shift})) << 5) + "
                f"static_cast<long long>(threadIdx.x & {lanes - 1}u) + {lanes} * hawk_q")

    @staticmethod
    def _reduce(k: int, width: int, code: str, lanes: int) -> str:
        fn = "rows_reduce_lanes" if lanes else "rows_reduce"
        return f"hk::ss::{fn}<{k}, {width}, {code}>(hawk_terms, hawk_ss_store);"

    def sample_sum_frame(self, width: int, elem: str, store: str,
                         op: str = "sum", live: str | None = None, elem_bytes: int = 8) -> tuple:
        """The row frame around a body writing ``width`` terms into ``hawk_ss``.

        A warp takes K consecutive rows per trip, loads of all K rows in flight
        together.  Where a row spreads over P = 32 / K lanes (``row_lanes``),
        lane l takes samples (l % P) + P q of row l / P and joins its own
        samples' tree levels in registers before the butterfly
        (hk::ss::rows_reduce_lanes); otherwise lane l takes sample 32 * row + l
        of each row and the K rows' columns are reduced in one halving
        butterfly (hk::ss::rows_reduce).  ``store`` is the body of
        ``hawk_ss_store(hawk_col, hawk_s, hawk_c)`` at row ``hawk_row``; a lane
        past ``count`` adds the identity."""
        if live is not None:
            raise HawkError("a sample sum over an active-set prefix is not built on the b200 target")
        code = _OP_CODE[op]
        k = self.fold_rows(width)
        lanes = self.row_lanes(k, elem_bytes)
        opened = (
            "    const long long hawk_rows = (count + 31) >> 5;\n"
            f"    for (long long hawk_r0 = hk::warp_first() * {k}; hawk_r0 < hawk_rows; "
            f"hawk_r0 += hk::warp_step() * {k}) {{\n"
            f"        {elem} hawk_terms[{k * width}];\n"
            "#pragma unroll\n"
            f"        for (int hawk_k = 0; hawk_k < {k * width}; ++hawk_k) hawk_terms[hawk_k] = "
            f"hk::ss::identity<{elem}>({code});\n"
            "#pragma unroll\n"
            f"        for (int hawk_q = 0; hawk_q < {k}; ++hawk_q) {{\n"
            f"        {elem}* const hawk_ss = hawk_terms + hawk_q * {width};\n"
            f"        const long long hawk_flat = {self._flat(lanes)};\n"
            "        if (hawk_flat < count) {\n"
            "        const long long hawk_i = base + hawk_flat;\n"
            "        const hk::SampleIndex i{hawk_i};\n"
            "        (void)hawk_i;\n"
            "        (void)nSamples;")
        closed = (
            "        }\n"
            "        }\n"
            f"{store.replace('__K__', str(k)).replace('__W__', str(width))}\n"
            f"        {self._reduce(k, width, code, lanes)}\n"
            "    }")
        return opened, closed

    def sample_sum_frame_staged(self, plan: StagePlan, width: int, elem: str, store: str,
                                op: str = "sum", elem_bytes: int = 8) -> tuple:
        """The row frame over tiles of 8 warps x K rows staged through shared
        memory: warp w of the CTA takes rows [w K, (w + 1) K) of each tile,
        its lanes mapped onto them as in ``sample_sum_frame``."""
        code = _OP_CODE[op]
        k = self.fold_rows(width)
        lanes = self.row_lanes(k, elem_bytes)
        span = 256 * k
        opened = "\n".join([
            "    const long long hawk_rows = (count + 31) >> 5;",
            plan.setup_lines(f"(hawk_rows + {8 * k - 1}) / {8 * k}", f"count / {span}",
                             f"(static_cast<long long>(blockIdx.x) + hk_jj * gridDim.x) * {span}"),
            plan.loop_head(),
            f"        const long long hawk_r0 = hk_t * {8 * k} + static_cast<long long>(threadIdx.x >> 5) * {k};",
            f"        {elem} hawk_terms[{k * width}];",
            "#pragma unroll",
            f"        for (int hawk_k = 0; hawk_k < {k * width}; ++hawk_k) hawk_terms[hawk_k] = "
            f"hk::ss::identity<{elem}>({code});",
            "#pragma unroll",
            f"        for (int hawk_q = 0; hawk_q < {k}; ++hawk_q) {{",
            f"        {elem}* const hawk_ss = hawk_terms + hawk_q * {width};",
            f"        const long long hawk_flat = {self._flat(lanes)};",
            "        if (hawk_flat < count) {",
            "        const long long hawk_i = base + hawk_flat;",
            f"        const hk::SampleIndex i{{hawk_i, hk_st, static_cast<int>(hawk_flat - hk_t * {256 * k})}};",
            "        (void)hawk_i;",
            "        (void)nSamples;",
        ])
        closed = "\n".join([
            "        }",
            "        }",
            "        if (hawk_r0 < hawk_rows) {",
            store.replace("__K__", str(k)).replace("__W__", str(width)),
            f"        {self._reduce(k, width, code, lanes)}",
            "        }",
            plan.loop_tail(),
        ])
        return opened, closed

    def sample_sum_frame_warp_tiled(self, plan: StagePlan, width: int, elem: str, store: str,
                                    op: str = "sum", elem_bytes: int = 8) -> tuple:
        """The row frame with each warp's next trip fetched while it reduces the
        current one: ``plan`` lays out one trip's inputs (32 K samples of every
        staged component) as the warp's own tile in the block's dynamic shared
        memory (hk::stage::WarpTile); lane 0 issues the next trip's bulk copies
        after the warp has read the current tile and before the butterfly.  A
        trip that is not a whole tile (the partition's last rows) or planes that
        are not 16-byte aligned are read from global memory, as in
        ``sample_sum_frame``, whose lane mapping and reduction this frame
        keeps."""
        code = _OP_CODE[op]
        k = self.fold_rows(width)
        lanes = self.row_lanes(k, elem_bytes)
        opened = "\n".join([
            "    const long long hawk_rows = (count + 31) >> 5;",
            "    extern __shared__ __align__(128) unsigned char hk_smem[];",
            f"    hk::stage::WarpTile hk_tile(hk_smem, {plan.stage_bytes}u, {plan.tx_bytes}u);",
            "    const bool hk_aligned = " + plan.aligned_test() + ";",
            "    auto hk_fill = [&](long long hk_r) {      // warp-uniform: the trip starting at row hk_r",
            f"        if (!hk_aligned || ((hk_r + {k}) << 5) > count) return;",
            "        hk_tile.fill([&](unsigned char* hk_to, unsigned long long* hk_bar) {",
            "            const long long hk_first = hk_r << 5;",
            *plan.copy_lines("            "),
            "        });",
            "    };",
            f"    const long long hk_step = hk::warp_step() * {k};",
            f"    long long hawk_r0 = hk::warp_first() * {k};",
            "    if (hawk_r0 < hawk_rows) hk_fill(hawk_r0);",
            "    for (; hawk_r0 < hawk_rows; hawk_r0 += hk_step) {",
            "        const unsigned char* const hk_st = hk_tile.acquire();",
            f"        {elem} hawk_terms[{k * width}];",
            "#pragma unroll",
            f"        for (int hawk_k = 0; hawk_k < {k * width}; ++hawk_k) hawk_terms[hawk_k] = "
            f"hk::ss::identity<{elem}>({code});",
            "#pragma unroll",
            f"        for (int hawk_q = 0; hawk_q < {k}; ++hawk_q) {{",
            f"        {elem}* const hawk_ss = hawk_terms + hawk_q * {width};",
            f"        const long long hawk_flat = {self._flat(lanes)};",
            "        if (hawk_flat < count) {",
            "        const long long hawk_i = base + hawk_flat;",
            "        const hk::SampleIndex i{hawk_i, hk_st, static_cast<int>(hawk_flat - (hawk_r0 << 5))};",
            "        (void)hawk_i;",
            "        (void)nSamples;",
        ])
        closed = "\n".join([
            "        }",
            "        }",
            "        if (hawk_r0 + hk_step < hawk_rows) hk_fill(hawk_r0 + hk_step);",
            store.replace("__K__", str(k)).replace("__W__", str(width)),
            f"        {self._reduce(k, width, code, lanes)}",
            "    }",
            "    hk_tile.finish();",
        ])
        return opened, closed

    def warp_tiled(self, plan: StagePlan, width: int, elem_bytes: int) -> bool:
        """Whether the row frame fetches each warp's next trip ahead
        (``sample_sum_frame_warp_tiled``): where the rows are spread over lanes
        (``row_lanes``) and eight warps' tiles fit WARP_TILE_MAX.  Measured on
        the float64 Param-gradient VJP at 2^26 samples, run after the forward
        as in the headline step: 0.2775 ms against 0.2907 (rows not spread,
        no fetch ahead) and 0.281-0.295 (spread, no fetch ahead)."""
        return bool(plan.views) and self.row_lanes(self.fold_rows(width), elem_bytes) != 0 and \
            128 + 8 * plan.stage_bytes <= WARP_TILE_MAX

    def dispatch(self, kind_spelling, branch_spellings, policy, **kw):
        """The per-node ``predicated``/``switch`` text: the reference's own,
        identical on every target (hawk/emit/wrapper.py:276-281)."""
        from hawk.emit.dispatch import render_dispatch_rank0
        return render_dispatch_rank0(kind_spelling, branch_spellings, policy, **kw)


#: Shared memory the stages of one CTA may take (the buffers; barriers aside).
STAGE_BUDGET = 96 * 1024
#: Largest stage set a CTA may take at all (two stages of a wide matrix plane).
STAGE_MAX = 200 * 1024
#: Largest block shared memory of the warp-tiled row frame (eight warps' tiles
#: and their barriers): three 256-thread blocks an SM still fit.
WARP_TILE_MAX = 64 * 1024


class StagePlan:
    """Which input components a CTA stages, where, and in how many stages.

    Staged are the per-sample inputs (``vec_in``, ``mat_in``, ``per_sample``),
    each component one contiguous run of ``tile`` samples per tile.  ``stages``
    is as many as fit STAGE_BUDGET, at least 2 and at most 4; a kernel whose two
    stages would pass STAGE_MAX is not staged."""

    def __init__(self, walk, elem_bytes: int, tile: int) -> None:
        sp = _spelling()
        self.tile = tile
        self.comp_bytes = tile * elem_bytes
        self.elem_bytes = elem_bytes
        self.views = []          # (binding, ncomps, rank)
        offset = 0
        self.offsets = {}
        for role, name in walk.arg_spec:
            if role not in ("vec_in", "mat_in", "per_sample"):
                continue
            shape = tuple(int(e) for e in walk.slot_types[(role, name)].shape)
            ncomp = 1
            for e in shape:
                ncomp *= e
            binding = sp.binding_name(role, name)
            self.views.append((binding, ncomp, len(shape)))
            self.offsets[(role, name)] = (offset, self.comp_bytes)
            offset += ncomp * self.comp_bytes
        self.tx_bytes = offset
        self.stage_bytes = -(-offset // 128) * 128
        fit = STAGE_BUDGET // self.stage_bytes if self.stage_bytes else 0
        self.stages = max(2, min(4, fit))
        self.enabled = bool(self.views) and self.stages * self.stage_bytes <= STAGE_MAX

    @property
    def smem_bytes(self) -> int:
        return 128 + self.stages * self.stage_bytes if self.enabled else 0

    def aligned_test(self) -> str:
        """Whether every staged component can be copied in tiles (16-byte
        aligned starts, pitches and partition base), as one C++ expression."""
        checks = []
        for binding, _ncomp, rank in self.views:
            pitch = f"{binding}.pitch * sizeof(*{binding}.data())" if rank else "0ull"
            checks.append(f"hk::stage::aligned({binding}.data(), {pitch}, base * "
                          f"static_cast<long long>(sizeof(*{binding}.data())))")
        return " && ".join(checks)

    def copy_lines(self, indent: str) -> list:
        """The bulk copies of one tile starting at sample ``base + hk_first``
        into ``hk_to``, counted on ``hk_bar``: one a component."""
        copies = []
        for binding, ncomp, rank in self.views:
            offset = self.offsets_by_binding[binding]
            for k in range(ncomp):
                src = (f"{binding}.data() + {k}ull * {binding}.pitch + base + hk_first" if rank
                       else f"{binding}.data() + base + hk_first")
                copies.append(f"{indent}hk::stage::copy(hk_to + {offset + k * self.comp_bytes}u, {src}, "
                              f"{self.comp_bytes}u, hk_bar);")
        return copies

    def setup_lines(self, tiles: str, full_tiles: str, first_of: str) -> str:
        """The pipe, the alignment test, the per-CTA tile counts and the
        copies of one tile (``hk_issue``), in the entry before its loop."""
        copies = self.copy_lines("        ")
        return "\n".join([
            "    extern __shared__ __align__(128) unsigned char hk_smem[];",
            f"    hk::stage::Pipe<{self.stages}> hk_pipe(hk_smem, {self.stage_bytes}u, {self.tx_bytes}u);",
            "    const bool hk_aligned = " + self.aligned_test() + ";",
            f"    const long long hk_tiles = {tiles};",
            "    const long long hk_mine = hk_tiles > static_cast<long long>(blockIdx.x)"
            " ? (hk_tiles - 1 - static_cast<long long>(blockIdx.x)) / gridDim.x + 1 : 0;",
            f"    const long long hk_full = {full_tiles};",
            "    const long long hk_staged = (!hk_aligned || hk_full <= static_cast<long long>(blockIdx.x)) ? 0"
            " : (hk_full - 1 - static_cast<long long>(blockIdx.x)) / gridDim.x + 1;",
            "    auto hk_issue = [&](long long hk_jj, unsigned char* hk_to, unsigned long long* hk_bar) {",
            f"        const long long hk_first = {first_of};",
            *copies,
            "    };",
            "    hk_pipe.setup(8u);",
            "    bool hk_ok = true;",
            "    if (threadIdx.x == 0)",
            f"        for (long long hk_jj = 0; hk_jj < {self.stages} && hk_jj < hk_staged && hk_ok; ++hk_jj)",
            "            hk_ok = hk_pipe.fill(hk_jj, [&](unsigned char* a, unsigned long long* b) { hk_issue(hk_jj, a, b); });",
            "    hk_ok = __shfl_sync(0xffffffffu, hk_ok, 0);",
        ])

    @property
    def offsets_by_binding(self) -> dict:
        sp = _spelling()
        return {sp.binding_name(r, n): off for (r, n), (off, _cb) in self.offsets.items()}

    def loop_head(self) -> str:
        return "\n".join([
            "    for (long long hk_j = 0; hk_j < hk_mine && hk_ok; ++hk_j) {",
            "        const long long hk_t = static_cast<long long>(blockIdx.x) + hk_j * gridDim.x;",
            "        const bool hk_use = hk_j < hk_staged;",
            "        const unsigned char* hk_st = nullptr;",
            "        if (hk_use) {",
            "            const unsigned char* hk_got = hk_pipe.acquire(hk_j);",
            "            if (!__all_sync(0xffffffffu, hk_got != nullptr)) break;",
            "            hk_st = hk_got;",
            "        }",
        ])

    def loop_tail(self) -> str:
        return "\n".join([
            "        if (hk_use) {",
            "            hk_pipe.release(hk_j);",
            f"            if (threadIdx.x == 0 && hk_j + {self.stages} < hk_staged)",
            f"                hk_ok = hk_pipe.fill(hk_j + {self.stages}, [&](unsigned char* a, unsigned long long* b) "
            f"{{ hk_issue(hk_j + {self.stages}, a, b); }});",
            "            hk_ok = __shfl_sync(0xffffffffu, hk_ok, 0);",
            "        }",
            "    }",
            "    if (threadIdx.x == 0) hk_pipe.drain();",
        ])


def lane_frame_staged(plan: StagePlan) -> tuple:
    """The lane frame over 256-sample tiles staged through shared memory:
    thread t takes sample t of each of its CTA's tiles."""
    opened = "\n".join([
        plan.setup_lines("(count + 255) >> 8", "count >> 8",
                         "(static_cast<long long>(blockIdx.x) + hk_jj * gridDim.x) << 8"),
        plan.loop_head(),
        "        const long long hawk_flat = (hk_t << 8) + static_cast<long long>(threadIdx.x);",
        "        if (hawk_flat < count) {",
        "        const long long hawk_i = base + hawk_flat;",
        "        const hk::SampleIndex i{hawk_i, hk_st, static_cast<int>(threadIdx.x)};",
        "        (void)hawk_i;",
        "        (void)nSamples;",
    ])
    closed = "\n".join(["        }", plan.loop_tail()])
    return opened, closed


def sample_sum_store(sums, banded: bool = False) -> str:
    """``hawk_ss_store``: butterfly column ``q * W + k`` is sink ``k``'s term of
    the trip's row ``q``; it goes to that sink's row plane (and its companion
    for a sum) at ``hawk_row``.  A row past the last is not stored.  ``__K__``
    and ``__W__`` are filled by the frame.  In the banded mode a sum's row is
    its compensated pair rounded once (``hawk_s + hawk_c``) and its companion
    row zero -- the reference's banded row is its accumulator's value and a
    zero companion (``ssOut_`` / ``ssComp_``, hawk/emit/wrapper.py:699-705)."""
    sp = _spelling()
    lines = ["        auto hawk_ss_store = [&](int hawk_col, auto hawk_s, auto hawk_c) {",
             "            (void)hawk_c;",
             "            const int hawk_q = hawk_col / __W__;",
             "            if (hawk_r0 + hawk_q >= hawk_rows) return;",
             "            const long long hawk_row = (base >> 5) + hawk_r0 + hawk_q;",
             "            hawk_col -= hawk_q * __W__;"]
    for k, sink in enumerate(sums):
        hi = sp.binding_name(sink.role, sink.name)
        lines.append(f"            {'else ' if k else ''}if (hawk_col == {k}) {{")
        if banded and sink.op == "sum":
            comp = sp.binding_name(sink.role, sink.companion.name)
            lines.append(f"                {hi}.data()[hawk_row] = hawk_s + hawk_c;")
            lines.append(f"                {comp}.data()[hawk_row] = static_cast<decltype(hawk_c)>(0);")
        else:
            lines.append(f"                {hi}.data()[hawk_row] = hawk_s;")
            if sink.op == "sum":
                comp = sp.binding_name(sink.role, sink.companion.name)
                lines.append(f"                {comp}.data()[hawk_row] = hawk_c;")
        lines.append("            }")
    return "\n".join(lines + ["        };"])


B200 = B200Wrapper()
