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
_SINK_ROLES = ("mutable", "out", "accum_out")
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


def view_decl(role: str, name: str, ttype) -> list:
    """The unpack lines of one slot: its view (or by-value local)."""
    sp = _spelling()
    ident = sp.binding_name(role, name)
    src = sp.param_name(role, name)
    elem = sp.element_spelling(ttype.dtype)
    shape = tuple(int(e) for e in ttype.shape)
    if role in _VALUE_ROLES:
        return [f"    const {param_type(role, ttype)} {ident} = {src};", f"    (void){ident};"]
    if role in _INPUT_ROLES:
        if len(shape) == 0:
            view = f"hk::ScalarIn<{elem}>"
        elif len(shape) == 1:
            view = f"hk::VecIn<{elem}, {shape[0]}>"
        elif len(shape) == 2:
            view = f"hk::MatIn<{elem}, {shape[0]}, {shape[1]}>"
        else:
            raise HawkError(f"slot {name!r}: a rank-{len(shape)} input plane is not built on the b200 target")
        return [f"    const {view} {ident}({src});", f"    (void){ident};"]
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

    def entry_signature(self, walk, name: str) -> str:
        """``extern "C" __global__`` entry: role mirrors by value in ``arg_spec``
        order, then the int64 partition triple."""
        sp = _spelling()
        params = [f"    {param_type(role, walk.slot_types[(role, n)])} {sp.param_name(role, n)}"
                  for role, n in walk.arg_spec]
        params += ["    long long base", "    long long count", "    long long nSamples"]
        return (f'extern "C" __global__ void __launch_bounds__({BLOCK}) {name}(\n'
                + ",\n".join(params) + ")")

    def index_prologue(self, segment=None, *, active=None, box=None, team=None) -> str:
        """The lane frame: a grid-stride loop binding ``hawk_i`` and ``i``."""
        for label, value in (("segmented", segment), ("active-set", active),
                             ("thread-box", box), ("team", team)):
            if value is not None:
                raise HawkError(f"the {label} entry is not built on the b200 target")
        return ("    for (long long hawk_flat = hk::lane_first(); hawk_flat < count; "
                "hawk_flat += hk::lane_step()) {\n"
                "        const long long hawk_i = base + hawk_flat;\n"
                "        const hk::SampleIndex i{hawk_i};\n"
                "        (void)hawk_i;\n"
                "        (void)nSamples;")

    def index_epilogue(self) -> str:
        return "    }"

    def unpack(self, walk) -> str:
        """Every slot's view, in ``arg_spec`` order; a promoted Param's one-cell
        plane is read once, ahead of the loop (hawk/emit/wrapper.py:1599-1605)."""
        sp = _spelling()
        lines = []
        for role, name in walk.arg_spec:
            ttype = walk.slot_types[(role, name)]
            lines += view_decl(role, name, ttype)
            if role == "lookup" and name in walk.param_planes:
                cell = sp.param_cell_binding(name)
                lines += [f"    const auto {cell} = {sp.binding_name(role, name)}.cell();",
                          f"    (void){cell};"]
        return "\n".join(lines)

    def fold_rows(self, width: int) -> int:
        """Rows one warp folds per trip: the largest power of two K with
        K * width <= 32 butterfly columns (hk::ss::rows_reduce).  Measured on
        the B200 for the 3-column Param-gradient VJP at 2^26 samples: K = 2, 4,
        8, 16 take 0.58, 0.57, 0.36, 0.53 ms; a shared-memory variant in which
        each lane evaluates one whole (row, column) tree took 0.375 ms."""
        k = 1
        while k < 32 and 2 * k * width <= 32:
            k *= 2
        return k

    def sample_sum_frame(self, width: int, elem: str, store: str,
                         op: str = "sum", live: str | None = None) -> tuple:
        """The row frame around a body writing ``width`` terms into ``hawk_ss``.

        A warp takes K consecutive rows per trip (lane l on sample 32 * row + l
        of each, loads of all K rows in flight together); the K rows' columns
        are reduced in one halving butterfly (hk::ss::rows_reduce).  ``store``
        is the body of ``hawk_ss_store(hawk_col, hawk_s, hawk_c)`` at row
        ``hawk_row``; a lane past ``count`` adds the identity."""
        if live is not None:
            raise HawkError("a sample sum over an active-set prefix is not built on the b200 target")
        code = _OP_CODE[op]
        k = self.fold_rows(width)
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
            "        const long long hawk_flat = ((hawk_r0 + hawk_q) << 5) + static_cast<long long>(threadIdx.x & 31u);\n"
            "        if (hawk_flat < count) {\n"
            "        const long long hawk_i = base + hawk_flat;\n"
            "        const hk::SampleIndex i{hawk_i};\n"
            "        (void)hawk_i;\n"
            "        (void)nSamples;")
        closed = (
            "        }\n"
            "        }\n"
            f"{store.replace('__K__', str(k)).replace('__W__', str(width))}\n"
            f"        hk::ss::rows_reduce<{k}, {width}, {code}>(hawk_terms, hawk_ss_store);\n"
            "    }")
        return opened, closed

    def dispatch(self, kind_spelling, branch_spellings, policy, **kw):
        """The per-node ``predicated``/``switch`` text: the reference's own,
        identical on every target (hawk/emit/wrapper.py:276-281)."""
        from hawk.emit.dispatch import render_dispatch_rank0
        return render_dispatch_rank0(kind_spelling, branch_spellings, policy, **kw)


def sample_sum_store(sums) -> str:
    """``hawk_ss_store``: butterfly column ``q * W + k`` is sink ``k``'s term of
    the trip's row ``q``; it goes to that sink's row plane (and its companion
    for a sum) at ``hawk_row``.  A row past the last is not stored.  ``__K__``
    and ``__W__`` are filled by the frame."""
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
        lines.append(f"                {hi}.data()[hawk_row] = hawk_s;")
        if sink.op == "sum":
            comp = sp.binding_name(sink.role, sink.companion.name)
            lines.append(f"                {comp}.data()[hawk_row] = hawk_c;")
        lines.append("            }")
    return "\n".join(lines + ["        };"])


B200 = B200Wrapper()
