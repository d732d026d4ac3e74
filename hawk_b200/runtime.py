"""Load and run b200 artifacts on device planes: the device twin of ``hawk.load`` / ``hawk.run``.

The reference's runtime (hawk/runtime.py:494-602) loads a host artifact,
validates every bound plane against the sidecar (hawk/_bind_checks.py:436),
binds each slot into an argument block and calls the entry once over
``[base, base + count)``; a kernel that reduces over samples into cells gets
its row scratch from the runtime, and the rows are finished into the caller's
cells (hawk/runtime.py:345-360, :588-602, hawk/_cells.py).

This module does the same for the b200 target, with device planes:

* ``load(directory, kernel, mode=..., device=...)`` loads ``<kernel>.<mode>.cubin``
  through the C ABI (which self-checks its exports) and builds the argument
  block from the sidecar's slot descriptors;
* ``run(kernel, **planes)`` validates and binds the planes (dtype, shape,
  device, contiguity, writability -- every failing argument named in one
  refusal), launches on the caller's stream and, for a kernel with cells,
  finishes the rows on the device into the cells: one launch folds every
  column's rows into leaf partials (``hkb_cells_leaves``), one folds the leaves
  (``hkb_cells_tree``).

Launches are asynchronous on the stream (the current torch stream of the
kernel's device unless ``stream=`` names one); the cells hold their values
when the stream reaches them.  One ``DeviceKernel`` shared by threads
serialises its bind+launch under its lock, as the reference's HostKernel does
(hawk/runtime.py:46-54).
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import threading
import warnings
from pathlib import Path

from . import abi
from .errors import HawkError
from .planes import Plane, as_plane

#: Roles whose plane's trailing extent is the sample count (they vote on n).
PER_SAMPLE_ROLES = ("mutable", "out", "vec_in", "mat_in", "per_sample", "terminated")
#: Roles that are written by the kernel (their plane must be writable).
SINK_ROLES = ("mutable", "out", "accum_out", "terminated")
#: The automatic kernel's trip-budget word (hawk/ir/nodes.py FUSED_STEPS_PLANE).
FUSED_STEPS = "fused_steps"
ROW = 32

#: The element type of each scalar mode's planes and cells (a banded value is
#: an IEEE binary64 in its 8-byte cell on the b200 target).
_WIRE_OF_MODE = {"float64": "float64", "float32": "float32", "banded": "float64"}
_INT_DTYPES = ("i32", "i64", "int32", "uint32")


def descriptor_for_sidecar(sidecar: dict) -> list:
    """The argument-block kind of every slot, in arg_spec order (the rule of
    the reference's ``kind_for``, hawk/runtime.py:96-118)."""
    mode = sidecar.get("scalar_type", "float64")
    kinds = []
    for slot in sidecar["b200"]["slots"]:
        role, dtype, shape = slot["role"], slot["dtype"], slot["shape"]
        if role == "nsamples":
            kinds.append("nsamples")
        elif role == "uniform":
            kinds.append("int" if dtype in _INT_DTYPES else ("f32" if mode == "float32" else "f64"))
        elif role in ("vec_in", "mat_in", "out") or (role == "mutable" and shape):
            kinds.append("gref")
        elif dtype in _INT_DTYPES:
            kinds.append("int_handle")
        else:
            kinds.append("handle")
    return kinds


def _box(kind: str, value):
    if kind == "f64":
        return ctypes.c_double(float(value))
    if kind == "f32":
        return ctypes.c_float(float(value))
    if kind in ("int", "nsamples"):
        return ctypes.c_longlong(int(value))
    raise HawkError(f"slot kind {kind!r} is not a by-value slot")


#: Bits of a unit's error word (hk/stage.cuh) and what each reports.
WAIT_FULL, WAIT_EMPTY, WAIT_DRAIN, WAIT_WARP = 1, 2, 4, 16
WAIT_ERRORS = {WAIT_FULL: "a staged input tile did not arrive within the wait limit",
               WAIT_EMPTY: "a shared-memory stage was not released within the wait limit",
               WAIT_DRAIN: "a block gave up with copies into shared memory still in flight",
               WAIT_WARP: "a warp's fetched-ahead input tile did not arrive within the wait limit "
                          "(the warp read those inputs from global memory instead)"}


class DeviceKernel:
    """One b200 artifact's entry on one device, self-checked at load."""

    def __init__(self, directory, kernel: str, mode: str = "float64", device: int | None = None,
                 sidecar: dict | None = None) -> None:
        self.directory = Path(directory)
        stem = f"{kernel}.{mode}"
        if sidecar is None:
            path = sidecar_path(self.directory, kernel, mode)
            if path is None:
                raise HawkError(f"no b200 artifact {stem!r} in {self.directory} (no {stem}.json, nor a "
                                f"{kernel}.json of scalar type {mode})")
            sidecar = json.loads(path.read_text())
        if "b200" not in sidecar:
            raise HawkError(f"{stem}: its sidecar carries no 'b200' block; it was not built for the b200 target")
        self.sidecar = sidecar
        self.name = sidecar["kernel"]
        self.mode = sidecar.get("scalar_type", mode)
        self.element = _WIRE_OF_MODE.get(self.mode, self.mode)
        b200 = sidecar["b200"]
        check_unit_digest(self.directory, b200)
        self.frame = b200["frame"]
        self.sums = b200["sample_sums"]
        self.slots = [(s["role"], s["name"], s["dtype"], tuple(s["shape"])) for s in b200["slots"]]
        self.arg_spec = tuple((r, n) for r, n, _d, _s in self.slots)
        self.cells = sidecar.get("cells") or {}
        # the accum_out planes that are sample-sum rows (the rest are scatter targets)
        self.row_planes = {x for sm in self.sums for x in (sm["name"], sm.get("companion")) if x}
        if device is None:
            device = _current_device()
        self.device = int(device)
        self.library = abi.Library(self.directory / b200["cubin"], self.device)
        self.entry = self.library.entry(b200["entry"])
        # an automatic stepping kernel's persistent entry (<name>_persist)
        self.persist = self.library.entry(b200["persist"]) if b200.get("persist") else None
        # and its contiguous-range entry (<name>_range)
        self.ranged = self.library.entry(b200["range"]) if b200.get("range") else None
        # the fold of each compensated scatter target's companion (<name>__fold_<target>)
        self.folds = {t: self.library.entry(e) for t, e in (b200.get("folds") or {}).items()}
        self.descriptor = descriptor_for_sidecar(sidecar)
        self.block = abi.ArgBlock(self.descriptor)
        self.poisoned = ""
        self._lock = threading.Lock()
        self._held: list = []
        self._scratch: dict = {}
        self.finished = None            # the finished_count cell a run bound by default
        self._one_step = None           # the fused_steps word of 1 a run bound by default

    # -- validation ---------------------------------------------------------
    def _wire(self, name: str, dtype: str) -> str:
        wire = self.sidecar.get("arg_dtypes", {}).get(name)
        if wire:
            # an index word rides 64 bits (hawk/runtime.py:221-225); a banded cell is a binary64 word
            return _WIRE_OF_MODE.get(wire, wire) if wire == "banded" else wire
        if dtype in _INT_DTYPES:
            return {"i32": "int32", "i64": "int64"}.get(dtype, dtype)
        return _WIRE_OF_MODE[self.mode]

    def own_companions(self, arrays: dict, stream=None) -> tuple:
        """``(arrays, owned)``: ``arrays`` plus a zeroed companion, the target's
        shape, for each compensated scatter target whose companion the caller
        left out -- the run owns it (hawk/runtime.py:516-528)."""
        import torch

        owned = {comp: target for comp, target in (self.sidecar.get("companions") or {}).items()
                 if comp not in arrays and target in arrays}
        if not owned:
            return arrays, owned
        extra = {}
        for comp, target in owned.items():
            t = arrays[target]
            if not torch.is_tensor(t):
                raise HawkError(f"kernel {self.name!r}: bind the companion {comp!r} of {target!r} (the runtime "
                                "makes one only beside a torch tensor target)")
            with torch.cuda.stream(_torch_stream(stream, self.device)):
                extra[comp] = torch.zeros_like(t)
        self._held.append(extra)
        return {**arrays, **extra}, owned

    def fold_companions(self, arrays: dict, owned: dict, stream=None) -> None:
        """Each owned companion into its target after the launch, through the
        unit's fold entry over the target's slots (hawk/runtime.py:531-540): the
        target then holds the compensated sum."""
        for target in owned.values():
            size = int(arrays[target].numel())
            self.folds[target].launch(self.block, 0, size, size, _stream(stream, self.device))

    def default_words(self, arrays: dict, stream=None) -> dict:
        """``arrays`` plus the reserved one-cell planes a runner normally binds,
        for each one this kernel declares and the caller leaves out
        (hawk/runtime.py:237-265): a ``fused_steps`` word of 1 (a launch
        outside a runner takes exactly one step) and a ``finished_count``
        counter reset to 0 (``self.finished`` holds it after the launch)."""
        import torch

        declared = {n for _r, n in self.arg_spec}
        counter = (self.sidecar.get("finish") or {}).get("counter")
        extra = {}
        dev = torch.device("cuda", self.device)
        if FUSED_STEPS in declared and FUSED_STEPS not in arrays:
            if getattr(self, "_one_step", None) is None:
                self._one_step = torch.ones(1, dtype=torch.int64, device=dev)
            extra[FUSED_STEPS] = self._one_step
        if counter and counter in declared and counter not in arrays:
            if getattr(self, "finished", None) is None:
                self.finished = torch.zeros(1, dtype=torch.uint32, device=dev)
            with torch.cuda.stream(_torch_stream(stream, self.device)):
                self.finished.zero_()
            extra[counter] = self.finished
        return {**arrays, **extra} if extra else arrays

    def n_from(self, planes: dict) -> int:
        """The sample count every bound per-sample plane agrees on."""
        votes = {}
        for role, name, _dtype, shape in self.slots:
            if role not in PER_SAMPLE_ROLES or name not in planes:
                continue
            p = planes[name]
            if len(p.shape) != len(shape) + 1:
                continue                    # refused with its shape by the checks
            votes[name] = p.shape[-1]
        if not votes:
            raise HawkError(f"kernel {self.name!r}: no bound per-sample plane to read the sample count "
                            "from; pass n_samples= explicitly")
        if len(set(votes.values())) != 1:
            raise HawkError(f"kernel {self.name!r}: the bound per-sample planes disagree on the sample "
                            f"count: {sorted(votes.items())} -- pass n_samples= explicitly")
        return next(iter(votes.values()))

    def check(self, planes: dict, values: dict, n: int, extents: dict | None = None) -> None:
        """Every slot against its declaration; one refusal naming every failure.
        ``extents`` gives the trailing extent a plane must hold where it is not
        ``n`` (a split stage's planes over keys or target cells)."""
        errors = []
        extents = extents or {}
        for role, name, dtype, shape in self.slots:
            if role == "nsamples":
                continue
            if role == "uniform":
                if name not in values:
                    errors.append(f"argument {name!r}: this kernel declares a 'uniform' slot for it, "
                                  "but no value was bound")
                elif dtype in _INT_DTYPES and isinstance(values[name], float):
                    errors.append(f"argument {name!r}: expected an int uniform, got a float value")
                continue
            if name not in planes:
                errors.append(f"argument {name!r}: this kernel declares a {role!r} slot for it, "
                              "but no plane was bound")
                continue
            p: Plane = planes[name]
            want = self._wire(name, dtype)
            if p.dtype != want:
                errors.append(f"argument {name!r}: expected dtype {want}, got {p.dtype}")
            if p.device is None:
                errors.append(f"argument {name!r}: a host array; the b200 path binds device planes only")
            elif p.device != self.device:
                errors.append(f"argument {name!r}: on device {p.device}, the kernel is loaded on "
                              f"device {self.device}")
            if not p.contiguous:
                errors.append(f"argument {name!r}: the plane is bound by address at computed sample "
                              "offsets, so it must be C-contiguous")
            if role in SINK_ROLES and p.readonly:
                errors.append(f"argument {name!r}: a {role!r} plane is written and must be writable")
            if role == "accum_out" and name in self.row_planes:
                rows = -(-n // ROW)
                if len(p.shape) != 1 or p.shape[0] < rows:
                    errors.append(f"argument {name!r}: a row plane of {rows} rows (one per 32 samples) "
                                  f"is expected, got shape {p.shape}")
            elif role == "accum_out":
                # a scattered commit's target: any number of slots, the key's range
                if len(p.shape) != len(shape) + 1 or tuple(p.shape[:-1]) != tuple(shape) or p.shape[-1] < 1:
                    errors.append(f"argument {name!r}: a scatter target of shape ({', '.join(map(str, shape))}"
                                  f"{', ' if shape else ''}slots) is expected, got {p.shape}")
            elif role == "lookup":
                if len(p.shape) != 1 or p.shape[0] < 1:
                    errors.append(f"argument {name!r}: a lookup plane is 1-D and non-empty, got shape {p.shape}")
            else:
                want_shape = (*shape, "L")
                if len(p.shape) != len(shape) + 1 or tuple(p.shape[:-1]) != tuple(shape):
                    errors.append(f"argument {name!r}: expected shape {want_shape} (samples last), "
                                  f"got {p.shape}")
                elif name in extents:
                    if p.shape[-1] < extents[name]:
                        errors.append(f"argument {name!r}: holds {p.shape[-1]} entries, fewer than the "
                                      f"{extents[name]} the stage writes")
                elif p.shape[-1] < n:
                    errors.append(f"argument {name!r}: holds {p.shape[-1]} samples, fewer than "
                                  f"n_samples={n}")
        errors += adjoint_errors(adjoint_like(self.slots), planes)
        if errors:
            if len(errors) == 1:
                raise HawkError(f"kernel {self.name!r}: {errors[0]}")
            raise HawkError(f"kernel {self.name!r}: {len(errors)} arguments failed validation:\n"
                            + "\n".join(f"  - {e}" for e in errors))

    # -- bind + launch ------------------------------------------------------
    def bind_all(self, planes: dict, values: dict, n: int) -> None:
        """Bind every slot (planes already validated)."""
        held = []
        for slot, (role, name, _dtype, _shape) in enumerate(self.slots):
            kind = self.descriptor[slot]
            if role == "nsamples":
                box = _box(kind, n)
                held.append(box)
                self.block.bind(slot, ctypes.addressof(box), n, 1, 1, 0)
            elif role == "uniform":
                box = _box(kind, values[name])
                held.append(box)
                self.block.bind(slot, ctypes.addressof(box), n, 1, 1, 0)
            else:
                p = planes[name]
                samples = p.shape[-1] if p.shape else 1
                self.block.bind(slot, p.ptr, samples, 1, 2, self.device)
                held.append(p.keep)
        self._held = held

    def launch(self, base: int, count: int, n_samples: int, stream: int | None = None) -> None:
        """The launch crossing over ``[base, base + count)`` of the bound planes.
        An entry that stages its inputs through shared memory waits on the
        copies with bounded waits: after its launch the stream is synchronised
        and the unit's error word checked (``check_waits``)."""
        if self.frame == "row" and base % ROW:
            raise HawkError(f"kernel {self.name!r} reduces over 32-sample rows, so a partition must "
                            f"start on a row (base % 32 == 0), got base={base}")
        if self.poisoned:
            raise HawkError(self.poisoned)
        s = _stream(stream, self.device)
        self.entry.launch(self.block, base, count, n_samples, s)
        if self.sidecar["b200"].get("stages"):
            _torch_stream(s, self.device).synchronize()
            self.check_waits()

    def check_waits(self) -> None:
        """Read and clear the unit's error word and refuse what it reports: a
        stage's copy that did not arrive, or a stage not released, within the
        wait limit (the launch's outputs are incomplete); a block that gave up
        with copies into shared memory still in flight (``kErrDrain``), after
        which this unit is not launched again in this process -- another block
        may have been given that shared memory while the copy was landing.  A
        warp-tiled entry's wait that ran out alone (``kErrWarpWait``) left the
        outputs complete -- the warp read global memory instead -- and is
        reported as a warning.  A staged entry is checked after every launch;
        a warp-tiled one, whose launches do not synchronise, when the caller
        calls this (a synchronising read of the word)."""
        flags = self.library.errors(clear=True)
        if not flags:
            return
        what = [text for bit, text in WAIT_ERRORS.items() if flags & bit]
        message = f"kernel {self.name!r}: {'; '.join(what) or f'error word {flags:#x}'}"
        if flags & WAIT_DRAIN:
            self.poisoned = (message + "; the unit is not launched again in this process (reload the "
                             "library in a new process)")
            raise HawkError(self.poisoned)
        if flags == WAIT_WARP:
            warnings.warn(message + "; the outputs are complete", RuntimeWarning, stacklevel=2)
            return
        raise HawkError(message + "; the launch's outputs are incomplete")

    def cells_state(self, n: int):
        """The kernel's own cell scratch at sample count ``n`` (made once per n):
        the row planes of every sink (and companion), the leaf partials of the
        finish (``(cols, leaves)`` each) and the finished column values."""
        import torch

        if n not in self._scratch:
            rows = -(-n // ROW)
            leaves = -(-rows // abi.LEAF_ROWS)
            dt = torch.float64 if self.element == "float64" else torch.float32
            dev = torch.device("cuda", self.device)
            planes = {}
            for s in self.sums:
                planes[s["name"]] = torch.empty(rows, dtype=dt, device=dev)
                if s["companion"]:
                    planes[s["companion"]] = torch.empty(rows, dtype=dt, device=dev)
            cols = max(len(self.sums), 1)
            self._scratch[n] = {"rows": planes,
                                "leaf_hi": torch.empty((cols, leaves), dtype=dt, device=dev),
                                "leaf_comp": torch.empty((cols, leaves), dtype=dt, device=dev),
                                "values": torch.empty(cols, dtype=dt, device=dev)}
        return self._scratch[n]

    def cells_leaves(self, state: dict, lo: int, hi: int, stream=None) -> int:
        """Rows ``[lo, hi)`` of every column folded into one partial per leaf
        (one launch for all columns); returns the leaf count."""
        itemsize = 8 if self.element == "float64" else 4
        op = self.sums[0]["op"] if self.sums else "sum"
        rows = state["rows"]
        his = [rows[s["name"]].data_ptr() + lo * itemsize for s in self.sums]
        comps = [rows[s["companion"]].data_ptr() + lo * itemsize for s in self.sums] if op == "sum" else None
        count = hi - lo
        leaves = -(-count // abi.LEAF_ROWS)
        leaf_hi, leaf_comp = state["leaf_hi"], state["leaf_comp"]
        # the partials of column k start at k * leaves (a (cols, leaves) view)
        abi.cells_leaves(op, self.element, his, comps, count, leaf_hi.data_ptr(), leaf_comp.data_ptr(),
                         _stream(stream, self.device))
        return leaves

    def cells_tree(self, leaf_hi, leaf_comp, leaves: int, values, stream=None) -> None:
        """The pairwise levels over ``leaves`` partials per column, into ``values``."""
        op = self.sums[0]["op"] if self.sums else "sum"
        abi.cells_tree(op, self.element, len(self.sums), leaf_hi.data_ptr(), leaf_comp.data_ptr(), leaves,
                       values.data_ptr(), _stream(stream, self.device))

    def write_cells(self, values, outputs: dict, stream=None) -> None:
        """The finished column values into the caller's cell planes."""
        import torch

        with torch.cuda.stream(_torch_stream(stream, self.device)):
            for k, s in enumerate(self.sums):
                keep = outputs[s["name"]].keep
                cell = keep if torch.is_tensor(keep) else torch.as_tensor(keep, device=f"cuda:{self.device}")
                cell.view(-1)[:1].copy_(values[k:k + 1])


def _torch_stream(stream, device: int):
    import torch

    if stream is None:
        return torch.cuda.current_stream(device)
    if isinstance(stream, torch.cuda.Stream):
        return stream
    return torch.cuda.ExternalStream(int(getattr(stream, "cuda_stream", stream)), device=device)


def _current_device() -> int:
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.current_device()
    except ImportError:                                 # pragma: no cover
        pass
    return 0


def _stream(stream, device: int) -> int:
    if stream is not None:
        return int(getattr(stream, "cuda_stream", stream))
    try:
        import torch
        return int(torch.cuda.current_stream(device).cuda_stream)
    except Exception:                                   # noqa: BLE001
        return 0


def adjoint_like(slots) -> dict:
    """``bar_<plane>`` to ``<plane>`` for each written plane that is the
    adjoint of a lookup plane (hawk/ir/walk.py:144-152): it must hold as many
    elements as that plane, since the kernel adds into it by the plane's own
    index, never by lane."""
    reads = {n for r, n, *_ in slots if r in ("lookup", "wide_in")}
    return {n: n[4:] for r, n, *_ in slots
            if r in ("accum_out", "wide_out") and n.startswith("bar_") and n[4:] in reads}


def adjoint_errors(like: dict, planes: dict) -> list:
    """A gradient plane smaller than the lookup plane it is the adjoint of
    (hawk/_bind_checks.py:384-395), one message each."""
    return [f"argument {grad!r}: the gradient of the lookup plane {plane!r} (shape {tuple(planes[plane].shape)}) "
            f"needs that many elements, got shape {tuple(planes[grad].shape)}"
            for grad, plane in like.items()
            if grad in planes and plane in planes and planes[grad].size < planes[plane].size]


class SplitKernel:
    """A kernel run as stages: the device twin of the reference runtime's
    ``_run_stages`` (hawk/runtime.py:699-748).  Its stages are the entries of
    one unit (hawk/ir/split.py cuts them):

    * a value reduced over samples and read later is finished between two
      stages: the stage that makes it runs the row frame into rows the runtime
      owns, the rows are finished on the device (the ordered tree of
      hawk/_cells.py, bit for bit) and every later stage that reads the cell
      binds it as a one-cell lookup plane; a cell the kernel also stores is
      copied into the caller's plane, one only a later stage reads is the
      kernel's own;
    * team-form linear algebra (hawk/ir/team.py) passes the lanes' matrices
      through scratch planes the runtime owns (``team_planes``: ``per_lane``
      elements per sample, made once per sample count, hawk/runtime.py:675-696),
      a team stage running one lane per warp.

    The stages launch in order on the stream."""

    def __init__(self, directory, kernel: str, mode: str = "float64", device: int | None = None) -> None:
        self.directory = Path(directory)
        stem = f"{kernel}.{mode}"
        path = self.directory / f"{stem}.json"
        if not path.exists():
            raise HawkError(f"no b200 artifact {stem!r} in {self.directory} (no {path.name})")
        sidecar = json.loads(path.read_text())
        self.sidecar = sidecar
        self.name = sidecar["kernel"]
        self.mode = sidecar.get("scalar_type", mode)
        self.element = _WIRE_OF_MODE.get(self.mode, self.mode)
        b200 = sidecar["b200"]
        check_unit_digest(self.directory, b200)
        self.device = int(device if device is not None else _current_device())
        self.team_planes = sidecar.get("team_planes") or {}
        self.keyed = sidecar.get("keyed") or {}
        self.lane_axes = [(a.get("label"), a.get("extent"))
                          for a in ((sidecar.get("launch") or {}).get("lane_space") or {}).get("axes", [])]
        self.cell_specs = sidecar.get("cells") or {}
        self.records = b200["split"]
        self.stages = []
        for st in self.records:
            stage_sidecar = {"kernel": st["entry"], "scalar_type": self.mode,
                             "cells": {c: self.cell_specs[c] for c in st.get("cells_out") or ()},
                             "arg_dtypes": {}, "b200": {"entry": st["entry"], "cubin": b200["cubin"],
                                                         "frame": st.get("kind", "lane"),
                                                         "sample_sums": st.get("sample_sums") or [],
                                                         "slots": st["slots"], "persist": None, "folds": {}}}
            if stage_sidecar["b200"]["frame"] == "team":
                stage_sidecar["b200"]["frame"] = "lane"
            self.stages.append(DeviceKernel(self.directory, st["entry"], self.mode, self.device,
                                            sidecar=stage_sidecar))
        self.slots = [(s["role"], s["name"], s["dtype"], tuple(s["shape"])) for s in b200["slots"]]
        self.arg_spec = tuple((r, n) for r, n, _d, _s in self.slots)
        # the cells a caller binds (one value per column); the rest are the kernel's own
        self.cells = {c: spec for c, spec in self.cell_specs.items() if not spec.get("internal")}
        self._lock = threading.Lock()
        self._scratch: dict = {}
        self._values: dict = {}

    #: The most lane chunks an ordered scatter adds in (hawk/_lane_bind.py:107-114).
    SCATTER_CHUNKS = 256

    @classmethod
    def scatter_chunks(cls, n: int, targets: int) -> int:
        """The chunks an ordered scatter of ``n`` lanes into ``targets`` cells adds in."""
        return min(cls.SCATTER_CHUNKS, max(1, n // max(targets, 1)))

    def team_units(self, spec: dict, n: int, sizes: dict) -> int:
        """Elements of a team plane per ``per_lane`` (hawk/_lane_bind.py:137-145):
        lanes, keys, one (``once``), or ``chunks * targets`` cells (``per_target``)."""
        if spec.get("once"):
            return 1
        if "per_target" in spec:
            size = sizes[spec["per_target"]]
            return self.scatter_chunks(n, size) * size
        if "keys" in spec:
            return self.keyed_size(spec["keys"], n) // int(spec["keys"].get("width", 1))
        return n

    def grid(self, record: dict, n: int, count: int, sizes: dict) -> int:
        """The teams a stage launches (hawk/_lane_bind.py:123-134): the
        partition's lanes, a block sum's keys (times its groups), an ordered
        scatter's lane chunks or its target's cells."""
        kind = record.get("grid", "lanes")
        if kind == "keys":
            keyed = record["keyed"]
            return self.keyed_size(keyed, n) // int(keyed.get("width", 1)) * int(record.get("groups") or 1)
        if kind == "chunks":
            # the b200 chunk stage walks each chunk with ``groups`` warps (one per key residue)
            return self.scatter_chunks(n, sizes[record["of"]]) * int(record.get("groups") or 1)
        if kind == "targets":
            return sizes[record["of"]]
        return count

    def scratch(self, n: int, sizes: dict | None = None, stream=None) -> dict:
        """The stages' scratch planes at ``n`` samples (and the ordered scatters'
        target sizes): made once per shape; a plane with a ``fill`` is refilled
        for every run, in stream order (hawk/runtime.py:675-696)."""
        import torch

        sizes = sizes or {}
        key = (n, tuple(sorted(sizes.items())))
        if key not in self._scratch:
            dev = torch.device("cuda", self.device)
            real = torch.float64 if self.element == "float64" else torch.float32
            self._scratch[key] = {
                name: torch.full((int(spec.get("per_lane", 1)) * self.team_units(spec, n, sizes),),
                                 spec.get("fill", 0),
                                 dtype=torch.int32 if spec.get("dtype") == "int32" else real, device=dev)
                for name, spec in self.team_planes.items()}
        planes = self._scratch[key]
        refill = [(planes[name], spec["fill"]) for name, spec in self.team_planes.items() if "fill" in spec]
        if refill:
            with torch.cuda.stream(_torch_stream(stream, self.device)):
                for t, value in refill:
                    t.fill_(value)
        return planes

    def keyed_size(self, spec: dict, n: int) -> int:
        """The elements of a keyed plane at ``n`` lanes: ``width`` payload
        entries over the kept lane axes, a runtime axis as long as the lane
        axis allows (hawk/_lane_bind.py:92-98)."""
        inner = 1
        for _label, extent in self.lane_axes[1:]:
            inner *= int(extent)
        runtime_extent = n // inner if self.lane_axes else n
        size = int(spec.get("width", 1))
        for _label, extent in spec.get("axes", []):
            size *= runtime_extent if extent is None else int(extent)
        return size

    def keyed_planes(self, n: int, stream=None) -> dict:
        """The keyed planes the stages pass between them (a sum over some lane
        axes read back at the lane's key) and their compensated companions:
        made once per sample count and zeroed for every run
        (hawk/runtime.py:655-673), in stream order."""
        import torch

        key = ("keyed", n)
        if key not in self._scratch:
            real = torch.float64 if self.element == "float64" else torch.float32
            dev = torch.device("cuda", self.device)
            planes = {}
            for name, spec in self.keyed.items():
                planes[name] = torch.empty(self.keyed_size(spec, n), dtype=real, device=dev)
                for stage in self.stages:
                    for comp, target in (stage.sidecar.get("companions") or {}).items():
                        if target == name:
                            planes[comp] = torch.empty_like(planes[name])
            self._scratch[key] = planes
        planes = self._scratch[key]
        with torch.cuda.stream(_torch_stream(stream, self.device)):
            for t in planes.values():
                t.zero_()
        return planes

    def block_outputs(self) -> dict:
        """The block sums' output planes a caller binds: ``{name: (payload, keyed)}``."""
        out = {}
        for record in self.records:
            if "ordered_fold" in (record.get("ops") or ()):
                continue            # an ordered gradient's fold stores into its table's gradient
            if record.get("grid") == "keys" and record.get("keyed"):
                for slot in record["slots"]:
                    if slot["role"] == "wide_out" and slot["name"] in {n for _r, n in self.arg_spec}:
                        out[slot["name"]] = (tuple(record["keyed"].get("payload") or ()), record["keyed"])
        return out

    def flat_block_outputs(self, arrays: dict, n: int) -> dict:
        """A block sum's output bound as ``(*payload, keys)`` (payload first,
        hawk/ir/team.py:591-600), checked and handed to its stage flat."""
        outs = self.block_outputs()
        if not outs:
            return arrays
        import torch

        arrays = dict(arrays)
        for name, (payload, keyed) in outs.items():
            if name not in arrays:
                continue
            t = arrays[name]
            keys = self.keyed_size(keyed, n) // int(keyed.get("width", 1))
            want = (*payload, keys)
            if not torch.is_tensor(t) or tuple(t.shape) != want or not t.is_contiguous():
                raise HawkError(f"kernel {self.name!r}: argument {name!r} is the per-key block sum, a contiguous "
                                f"device tensor of shape {want} (payload first, one per key), got "
                                f"{tuple(getattr(t, 'shape', ()))}")
            arrays[name] = t.reshape(-1)
        return arrays

    def cell_values(self) -> dict:
        """One device plane per cell (its columns), where a finished cell lives
        for the stages that read it."""
        import torch

        if not self._values:
            real = torch.float64 if self.element == "float64" else torch.float32
            self._values = {c: torch.empty(int(spec.get("columns", 1)), dtype=real,
                                           device=torch.device("cuda", self.device))
                            for c, spec in self.cell_specs.items()}
        return self._values

    def run(self, *, base: int = 0, count: int | None = None, n_samples: int | None = None, stream=None,
            **arrays) -> None:
        import torch

        from .planes import from_torch

        declared = {n for r, n in self.arg_spec if r != "nsamples"} | set(self.cells)
        unknown = sorted(set(arrays) - declared)
        if unknown:
            raise HawkError(f"kernel {self.name!r}: {unknown} are not planes it declares "
                            f"(declared: {sorted(declared)})")
        missing = sorted(declared - set(arrays))
        if missing:
            raise HawkError(f"kernel {self.name!r}: {missing} are declared but not bound")
        uniforms = {n for r, n in self.arg_spec if r == "uniform"}
        values = {k: v for k, v in arrays.items() if k in uniforms}
        if n_samples is None:
            n_samples = self.stages[0].n_from({k: as_plane(k, v) for k, v in arrays.items()
                                               if k not in uniforms and k not in self.block_outputs()})
        arrays = self.flat_block_outputs(arrays, n_samples)
        planes = {k: as_plane(k, v) for k, v in arrays.items() if k not in uniforms}
        errors = adjoint_errors(adjoint_like(self.slots), planes)
        if errors:
            raise HawkError(f"kernel {self.name!r}: " + "; ".join(errors))
        for c, spec in self.cells.items():
            p = planes[c]
            if p.dtype != self.element or p.device != self.device or p.size < int(spec.get("columns", 1)):
                raise HawkError(f"kernel {self.name!r}: cell {c!r} must be a {self.element} plane of "
                                f"{spec.get('columns', 1)} value(s) on device {self.device}, got {p.dtype} "
                                f"{p.shape} on {p.device}")
        count = n_samples - base if count is None else count
        if base < 0 or count < 0 or base + count > n_samples:
            raise HawkError(f"kernel {self.name!r}: partition [{base}, {base + count}) is outside "
                            f"the {n_samples} samples")
        if self.cell_specs and base % ROW:
            raise HawkError(f"kernel {self.name!r} reduces over 32-sample rows, so a partition must "
                            f"start on a row (base % 32 == 0), got base={base}")
        # the cells an ordered scatter adds into: the bound target plane's elements
        sizes = {r["of"]: planes[r["of"]].size for r in self.records if r.get("of") and r["of"] in planes}
        with self._lock:
            owned = self.scratch(n_samples, sizes, stream)
            scratch = {k: from_torch(v) for k, v in owned.items()}
            scratch.update({k: from_torch(v) for k, v in self.keyed_planes(n_samples, stream).items()})
            cells = self.cell_values()
            for stage, record in zip(self.stages, self.records):
                names = {n for _r, n in stage.arg_spec}
                bound = {k: v for k, v in planes.items() if k in names and k not in self.cells}
                bound.update({k: v for k, v in scratch.items() if k in names})
                for cell in record.get("cells_in") or ():
                    cols = int(self.cell_specs[cell].get("columns", 1))
                    plane_names = (cell,) if cols == 1 else tuple(f"{cell}_{k}" for k in range(cols))
                    for k, plane in enumerate(plane_names):
                        bound[plane] = from_torch(cells[cell][k:k + 1])
                state = None
                if record.get("cells_out"):
                    state = stage.cells_state(n_samples)
                    bound.update({k: from_torch(v) for k, v in state["rows"].items()})
                if record.get("grid", "lanes") != "lanes":
                    # a stage over keys, lane chunks or target cells: its teams span the whole run
                    teams = self.grid(record, n_samples, count, sizes)
                    if teams == 0:
                        continue            # an ordered scatter into no cells adds nothing
                    # per-sample planes hold the run's lanes; scratch holds its own units; a
                    # block sum's output one entry a key; an ordered scatter's target its cells
                    keys = teams // int(record.get("groups") or 1) if record["grid"] == "keys" else 0
                    extents = {name: 0 for name in scratch}
                    extents.update({name: keys for role, name in stage.arg_spec
                                    if role == "wide_out" and name not in scratch})
                    stage.check(bound, values, n_samples, extents)
                    stage.bind_all(bound, values, n_samples)
                    stage.launch(0, teams, n_samples, stream)
                else:
                    # scratch planes are sized by their units (lanes, keys, once), not checked by lane
                    stage.check(bound, values, n_samples, {name: 0 for name in scratch})
                    stage.bind_all(bound, values, n_samples)
                    stage.launch(base, count, n_samples, stream)
                if state is None:
                    continue
                lo, hi = base // ROW, -(-(base + count) // ROW)
                sums = [s["name"] for s in stage.sums]
                if hi > lo:
                    leaves = stage.cells_leaves(state, lo, hi, stream)
                    stage.cells_tree(state["leaf_hi"], state["leaf_comp"], leaves, state["values"], stream)
                with torch.cuda.stream(_torch_stream(stream, self.device)):
                    for cell in record["cells_out"]:
                        cols = int(self.cell_specs[cell].get("columns", 1))
                        plane_names = (cell,) if cols == 1 else tuple(f"{cell}_{k}" for k in range(cols))
                        for k, plane in enumerate(plane_names):
                            cells[cell][k:k + 1].copy_(state["values"][sums.index(plane):sums.index(plane) + 1])
                        if cell in self.cells:
                            keep = planes[cell].keep
                            out = keep if torch.is_tensor(keep) else torch.as_tensor(keep, device=f"cuda:{self.device}")
                            out.view(-1)[:cols].copy_(cells[cell])
            for record in self.records:
                status = record.get("status")
                if status and status in owned:
                    # an ordered scatter's key outside [0, cells) other than -1 is refused by
                    # name after the run (hawk/_lane_bind.py:148-154): the flags from element 1
                    flags = owned[status][1:]
                    if bool(torch.any(flags != 0).item()):
                        raise HawkError(f"{self.name}: hawk.scatter({record['of']}, policy='ordered') got a key "
                                        f"outside [0, {sizes.get(record['of'])}) that is not the skip key -1; those "
                                        f"adds were dropped, the rest are in {record['of']}")

    def errors(self, clear: bool = True) -> int:
        """The unit's error word (hkb_library_errors) after the stream's launches."""
        flags = 0
        for stage in self.stages:
            flags |= stage.library.errors(clear)
        return flags


_CACHE: dict = {}
_CACHE_LOCK = threading.Lock()


def check_unit_digest(directory, b200: dict) -> None:
    """Refuse an artifact whose unit beside it no longer has the digest its
    sidecar records: the CUBIN and the sidecar's slot records may then be of
    another unit (a unit edited or re-rendered without its sidecar)."""
    unit = Path(directory) / b200.get("unit", "")
    want = b200.get("unit_digest")
    if want and unit.is_file():
        got = hashlib.sha256(unit.read_bytes()).hexdigest()
        if got != want:
            raise HawkError(f"{unit.name} is stale against its sidecar: the unit hashes to {got[:16]}..., "
                            f"the sidecar records {want[:16]}...; rebuild the artifact")


def sidecar_path(directory, kernel: str, mode: str):
    """The sidecar of ``kernel`` in ``mode``: ``<kernel>.<mode>.json`` (this
    build's bundles), else the reference's ``<kernel>.json`` when it records
    that scalar type (a bundle the reference's ``hawk.build`` wrote for the
    b200 row); None when neither is there."""
    directory = Path(directory)
    path = directory / f"{kernel}.{mode}.json"
    if path.exists():
        return path
    path = directory / f"{kernel}.json"
    if path.exists() and json.loads(path.read_text()).get("scalar_type", "float64") == mode:
        return path
    return None


def load(directory, kernel: str, mode: str = "float64", device: int | None = None):
    """Load ``kernel``'s b200 artifact in scalar mode ``mode`` from ``directory``
    on ``device`` (cached per process): a ``DeviceKernel``, or a ``SplitKernel``
    for a kernel built as stages."""
    key = (str(Path(directory).resolve()), kernel, mode, device if device is not None else _current_device())
    with _CACHE_LOCK:
        if key not in _CACHE:
            path = sidecar_path(directory, kernel, mode)
            split = path is not None and "split" in json.loads(path.read_text()).get("b200", {})
            _CACHE[key] = (SplitKernel if split else DeviceKernel)(directory, kernel, mode, key[3])
        return _CACHE[key]


def launch_cells(kernel: DeviceKernel, *, base: int = 0, count: int | None = None,
                 n_samples: int | None = None, stream=None, persist: dict | None = None,
                 ranged: dict | None = None, **arrays):
    """Validate, bind and launch (the body of ``run``); for a kernel with cells,
    return ``(state, outputs, lo_row, hi_row)`` for the caller to finish, else None.
    ``persist`` launches the persistent entry instead, with those keyword
    arguments of ``abi.Entry.launch_persist``; ``ranged`` the range entry, with
    those of ``abi.Entry.launch_range``."""
    arrays = kernel.default_words(arrays, stream)
    declared = {name for _r, name in kernel.arg_spec} | set(kernel.cells)
    unknown = sorted(set(arrays) - declared)
    if unknown:
        raise HawkError(f"kernel {kernel.name!r}: {unknown} are not planes it declares "
                        f"(declared: {sorted(declared)})")
    values = {}
    planes = {}
    uniforms = {n for r, n in kernel.arg_spec if r == "uniform"}
    for name, obj in arrays.items():
        if name in uniforms:
            values[name] = obj
        else:
            planes[name] = as_plane(name, obj)
    cells = kernel.cells
    if cells:
        rows_bound = [c for c in cells if c in planes and planes[c].size > 1]
        missing = [c for c in cells if c not in planes]
        if missing or rows_bound:
            raise HawkError(f"kernel {kernel.name!r}: this kernel reduces over samples into the cells "
                            f"{sorted(cells)}; bind each cell (one value per column), not its rows"
                            + (f" (missing: {missing})" if missing else ""))
    if n_samples is None:
        n_samples = kernel.n_from(planes)
    count = n_samples - base if count is None else count
    if base < 0 or count < 0 or base + count > n_samples:
        raise HawkError(f"kernel {kernel.name!r}: partition [{base}, {base + count}) is outside "
                        f"the {n_samples} samples")
    outputs = {}
    state = None
    if cells:
        for c in cells:
            p = planes[c]
            if p.dtype != kernel.element or p.device != kernel.device:
                raise HawkError(f"kernel {kernel.name!r}: cell {c!r} must be a {kernel.element} plane on device "
                                f"{kernel.device}, got {p.dtype} on {p.device}")
            outputs[c] = p
        state = kernel.cells_state(n_samples)
        from .planes import from_torch
        bound = {k: v for k, v in planes.items() if k not in cells}
        bound.update({k: from_torch(v) for k, v in state["rows"].items()})
    else:
        bound = planes
    kernel.check(bound, values, n_samples)
    kernel.bind_all(bound, values, n_samples)
    if persist is not None:
        kernel.persist.launch_persist(kernel.block, base, count, n_samples,
                                      stream=_stream(stream, kernel.device), **persist)
        return None
    if ranged is not None:
        kernel.ranged.launch_range(kernel.block, base, count, n_samples, stream=_stream(stream, kernel.device),
                                   **ranged)
        return None
    kernel.launch(base, count, n_samples, stream)
    if not cells:
        return None
    return state, outputs, base // ROW, -(-(base + count) // ROW)


#: Step cost (64-bit floating-point operations) from which the persistent entry
#: claims every 4 trips instead of every 32.  Measured on the B200: the RK4
#: oscillator (~30 per step) took 1.93 / 3.30 / 11.7 ms at chunks 32 / 4 / 1
#: (claims cost more than idle lanes), the Fehlberg 7(8) orbit (~1000 per step)
#: 4.24 / 3.20 / 3.57 ms (a finished lane idling to the chunk's end costs more).
HEAVY_STEP_FP64_OPS = 256


def default_chunk(kernel: DeviceKernel) -> int:
    """Trips between claims for ``kernel``'s persistent entry (see HEAVY_STEP_FP64_OPS)."""
    ops = kernel.sidecar["b200"].get("step_fp64_ops") or 0
    return 4 if ops >= HEAVY_STEP_FP64_OPS else 32


def run_persist(kernel: DeviceKernel, *, base: int = 0, count: int | None = None,
                n_samples: int | None = None, chunk: int | None = None, grid: int = 0, steps=None, stepsum=None,
                util=None, stream=None, **arrays):
    """Run an automatic stepping kernel's persistent entry over ``[base, base + count)``.

    Each sample runs to its finish or the ``fused_steps`` budget (a word of 1
    when left out), exactly as one launch of the kernel's own entry with that
    word would run it; lanes claim samples off a fresh counter, ``chunk``
    trips between claims.  ``steps`` (uint32, one cell), ``stepsum`` (uint64)
    and ``util`` (two uint64) receive the longest per-sample trip count, the
    steps run and the slot fill when given (each zeroed by the caller).  The
    finished counter -- bound, or ``kernel.finished`` -- holds the batch's
    finished count afterwards, samples finished on entry included.  Returns
    the claim counter (a device uint32).  ``chunk`` defaults by the step's cost
    (``default_chunk``)."""
    import torch

    if kernel.persist is None:
        raise HawkError(f"kernel {kernel.name!r} is not an automatic stepping kernel; it has no persistent entry")
    if chunk is None:
        chunk = default_chunk(kernel)
    if chunk < 0:
        raise HawkError(f"chunk={chunk}: the trips between claims is a count (0: whole samples)")
    for label, t, dtype, cells in (("steps", steps, torch.uint32, 1), ("stepsum", stepsum, torch.uint64, 1),
                                   ("util", util, torch.uint64, 2)):
        if t is not None and (not torch.is_tensor(t) or t.dtype != dtype or t.numel() < cells
                              or t.device != torch.device("cuda", kernel.device)):
            raise HawkError(f"{label}=: a device {dtype} tensor of {cells} cell(s) on cuda:{kernel.device}")
    with kernel._lock:
        claim = torch.zeros(1, dtype=torch.uint32, device=torch.device("cuda", kernel.device))
        with torch.cuda.stream(_torch_stream(stream, kernel.device)):
            claim.zero_()
        ptr = lambda t: 0 if t is None else t.data_ptr()   # noqa: E731
        launch_cells(kernel, base=base, count=count, n_samples=n_samples, stream=stream,
                     persist={"next_ptr": claim.data_ptr(), "util": ptr(util), "steps": ptr(steps),
                              "stepsum": ptr(stepsum), "chunk": chunk, "grid": grid}, **arrays)
        kernel._held.append(claim)
    return claim


def _report_cells(kernel, **cells) -> None:
    import torch

    for label, (t, dtype, n) in cells.items():
        if t is not None and (not torch.is_tensor(t) or t.dtype != dtype or t.numel() < n
                              or t.device != torch.device("cuda", kernel.device)):
            raise HawkError(f"{label}=: a device {dtype} tensor of {n} cell(s) on cuda:{kernel.device}")


def run_range(kernel: DeviceKernel, *, base: int = 0, count: int | None = None, n_samples: int | None = None,
              steps=None, stepsum=None, stream=None, **arrays) -> None:
    """Run an automatic stepping kernel's contiguous-range entry over ``[base, base + count)``.

    The same bits as ``run`` with the same ``fused_steps`` word; ``steps``
    (uint32, one cell) and ``stepsum`` (uint64) receive the longest per-sample
    step count of the launch and the steps run, when given (each zeroed by the
    caller).  The finished counter holds the batch's finished count afterwards,
    samples finished on entry included (hawk/emit/cuda.py:373-380)."""
    import torch

    if getattr(kernel, "ranged", None) is None:
        raise HawkError(f"kernel {kernel.name!r} is not an automatic stepping kernel; it has no range entry")
    _report_cells(kernel, steps=(steps, torch.uint32, 1), stepsum=(stepsum, torch.uint64, 1))
    ptr = lambda t: 0 if t is None else t.data_ptr()   # noqa: E731
    with kernel._lock:
        launch_cells(kernel, base=base, count=count, n_samples=n_samples, stream=stream,
                     ranged={"steps": ptr(steps), "stepsum": ptr(stepsum)}, **arrays)


def run(kernel: DeviceKernel, *, base: int = 0, count: int | None = None, n_samples: int | None = None,
        stream=None, **arrays) -> None:
    """Bind ``arrays`` and run the whole range in one launch (asynchronous on ``stream``).

    ``count`` defaults to ``n_samples``, ``n_samples`` to the count every bound
    per-sample plane agrees on.  A kernel with cells takes each cell as a
    one-element device plane (not its rows, as hawk/runtime.py:345-360 rules);
    the runtime owns the rows and finishes them on the device: one leaf launch
    and one tree launch for all columns.  A kernel built as stages runs them
    in order (``SplitKernel.run``)."""
    if isinstance(kernel, SplitKernel):
        kernel.run(base=base, count=count, n_samples=n_samples, stream=stream, **arrays)
        return
    with kernel._lock:
        arrays, owned = kernel.own_companions(arrays, stream)
        pending = launch_cells(kernel, base=base, count=count, n_samples=n_samples, stream=stream, **arrays)
        if owned:
            kernel.fold_companions(arrays, owned, stream)
        if pending is None:
            return
        state, outputs, lo, hi = pending
        if hi > lo:
            leaves = kernel.cells_leaves(state, lo, hi, stream)
            kernel.cells_tree(state["leaf_hi"], state["leaf_comp"], leaves, state["values"], stream)
            kernel.write_cells(state["values"], outputs, stream)
