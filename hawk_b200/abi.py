"""ctypes binding of libhawk_b200 (include/hawk_b200.h).

The in-tree library ``hawk_b200/lib/libhawk_b200.so`` is the only native code
this module loads; when it is missing the import of the runtime fails loudly
(build it with ``python -m hawk_b200.csrc.build``).  There is no fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .errors import HawkError

LIBRARY_PATH = Path(__file__).resolve().parent / "lib" / "libhawk_b200.so"

OK = 0
OP = {"sum": 0, "mean": 0, "max": 1, "min": 2}
DTYPE = {"float64": 0, "float32": 1}
LEAF_ROWS = 4096

#: Every symbol include/hawk_b200.h declares, with (restype, argtypes).
_c = ctypes
_P = _c.c_void_p
SIGNATURES = {
    "hkb_last_error": (_c.c_char_p, []),
    "hkb_build_digest": (_c.c_char_p, []),
    "hkb_layout_sizes": (_c.c_int, [_c.POINTER(_c.c_uint64)]),
    "hkb_device_count": (_c.c_int, [_c.POINTER(_c.c_int)]),
    "hkb_library_load": (_c.c_int, [_P, _c.c_size_t, _c.c_int, _c.POINTER(_P)]),
    "hkb_library_load_file": (_c.c_int, [_c.c_char_p, _c.c_int, _c.POINTER(_P)]),
    "hkb_library_free": (None, [_P]),
    "hkb_library_errors": (_c.c_int, [_P, _c.POINTER(_c.c_uint), _c.c_int]),
    "hkb_library_entry": (_c.c_int, [_P, _c.c_char_p, _c.POINTER(_P)]),
    "hkb_entry_info": (_c.c_int, [_P, _c.POINTER(_c.c_int), _c.POINTER(_c.c_int), _c.POINTER(_c.c_int),
                                  _c.c_int64, _c.POINTER(_c.c_int64)]),
    "hkb_argblock_create": (_c.c_int, [_c.POINTER(_c.c_char_p), _c.c_size_t, _c.POINTER(_P)]),
    "hkb_argblock_free": (None, [_P]),
    "hkb_argblock_bind": (_c.c_int, [_P, _c.c_size_t, _c.c_size_t, _c.c_uint64, _c.c_uint64,
                                     _c.c_int32, _c.c_int32]),
    "hkb_argblock_rebind": (_c.c_int, [_P, _c.POINTER(_c.c_int64), _c.POINTER(_c.c_int64), _c.c_size_t]),
    "hkb_entry_launch": (_c.c_int, [_P, _P, _c.c_int64, _c.c_int64, _c.c_int64, _P]),
    "hkb_entry_launch_persist": (_c.c_int, [_P, _P, _c.c_int64, _c.c_int64, _c.c_int64, _P, _P, _P, _P,
                                            _c.c_uint32, _c.c_int64, _P]),
    "hkb_entry_launch_range": (_c.c_int, [_P, _P, _c.c_int64, _c.c_int64, _c.c_int64, _P, _P, _P]),
    "hkb_cells_leaves": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _c.POINTER(_P), _c.POINTER(_P),
                                    _c.c_int64, _P, _P, _P]),
    "hkb_cells_tree": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _P, _P, _c.c_int64, _P, _P]),
    "hkb_cells_tree_ex": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _P, _P, _c.c_int64, _c.c_int64, _c.c_int64,
                                     _P, _P, _P]),
    "hkb_cells_scratch_bytes": (_c.c_size_t, [_c.c_int, _c.c_int, _c.c_int64]),
    "hkb_cells_finish": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _c.POINTER(_P), _c.POINTER(_P),
                                    _c.c_int64, _P, _P, _P]),
    "hkb_cells_finish_noalloc": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _c.POINTER(_P), _c.POINTER(_P),
                                            _c.c_int64, _P, _P]),
    "hkb_peer_create": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.POINTER(_P), _P]),
    "hkb_peer_connect": (_c.c_int, [_P, _P]),
    "hkb_peer_finish": (_c.c_int, [_P, _c.c_int, _P, _P, _c.c_int64, _P, _c.c_uint64, _c.c_uint64, _P]),
    "hkb_peer_status": (_c.c_int, [_P, _c.POINTER(_c.c_uint)]),
    "hkb_peer_free": (None, [_P]),
}

PEER_HANDLE_BYTES = 64
PEER_MAX_RANKS = 8
PEER_TIMEOUT = 1

_LOCK = threading.Lock()
_LIB = None


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once; raises when it is not built)."""
    global _LIB
    with _LOCK:
        if _LIB is None:
            if not LIBRARY_PATH.exists():
                raise HawkError(f"{LIBRARY_PATH.name} is not built (expected at {LIBRARY_PATH}); "
                                "build it with `python -m hawk_b200.csrc.build`")
            handle = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            check_build_digest(handle.hkb_build_digest().decode(), sources_digest())
            _LIB = handle
        return _LIB


def sources_digest():
    """The digest of the library's sources beside the package (the digest its
    build stamps in, ``hawk_b200.csrc.build.source_digest``), or None where the
    sources are not shipped."""
    try:
        from .csrc import build
    except ImportError:
        return None
    if not all(p.exists() for p in build.SOURCES + build.HEADERS):
        return None
    return build.source_digest()


def check_build_digest(built: str, sources) -> None:
    """Refuse a library built from other sources than the ones beside it (the
    reference refuses a stale extension the same way at import,
    hawk/__init__.py:128-209): its kernels and ABI would not be the ones the
    headers and units here declare."""
    if sources is not None and built != sources:
        raise HawkError(f"{LIBRARY_PATH.name} is stale: it was built from sources whose digest is "
                        f"{built[:16]}..., the sources beside it now hash to {sources[:16]}...; "
                        "rebuild it with `python -m hawk_b200.csrc.build`")


def check(status: int, what: str) -> None:
    if status != OK:
        msg = lib().hkb_last_error().decode(errors="replace")
        raise HawkError(f"{what}: {msg} (status {status})")


def layout_sizes() -> list:
    out = (ctypes.c_uint64 * 5)()
    check(lib().hkb_layout_sizes(out), "hkb_layout_sizes")
    return [int(v) for v in out]


def build_digest() -> str:
    return lib().hkb_build_digest().decode()


def device_count() -> int:
    n = ctypes.c_int(0)
    check(lib().hkb_device_count(ctypes.byref(n)), "hkb_device_count")
    return int(n.value)


class Library:
    """A loaded sm_100a artifact (``hawk._core.HostLibrary``'s device twin)."""

    def __init__(self, path, device: int) -> None:
        self._h = ctypes.c_void_p()
        self.path = Path(path)
        self.device = int(device)
        check(lib().hkb_library_load_file(str(self.path).encode(), self.device, ctypes.byref(self._h)),
              f"loading {self.path.name} on device {self.device}")

    def entry(self, name: str) -> "Entry":
        return Entry(self, name)

    def errors(self, clear: bool = True) -> int:
        """The unit's error word (0: every bounded device wait completed)."""
        flags = ctypes.c_uint(0)
        check(lib().hkb_library_errors(self._h, ctypes.byref(flags), 1 if clear else 0), "hkb_library_errors")
        return int(flags.value)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and h.value and _LIB is not None:
            _LIB.hkb_library_free(h)
            self._h = None


class Entry:
    def __init__(self, library: Library, name: str) -> None:
        self.library = library       # keeps the image loaded
        self.name = name
        self._h = ctypes.c_void_p()
        check(lib().hkb_library_entry(library._h, name.encode(), ctypes.byref(self._h)),
              f"entry {name!r} of {library.path.name}")

    def info(self, count: int = 0) -> dict:
        regs, bps, block = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        grid = ctypes.c_int64()
        check(lib().hkb_entry_info(self._h, ctypes.byref(regs), ctypes.byref(bps), ctypes.byref(block),
                                   int(count), ctypes.byref(grid)), "hkb_entry_info")
        return {"regs": regs.value, "blocks_per_sm": bps.value, "block": block.value, "grid": grid.value}

    def launch(self, block: "ArgBlock", base: int, count: int, n_samples: int, stream: int = 0) -> None:
        check(lib().hkb_entry_launch(self._h, block._h, int(base), int(count), int(n_samples),
                                     ctypes.c_void_p(int(stream) or None)),
              f"launching {self.name!r}")

    def launch_persist(self, block: "ArgBlock", base: int, count: int, n_samples: int, next_ptr: int,
                       util: int = 0, steps: int = 0, stepsum: int = 0, chunk: int = 32, grid: int = 0,
                       stream: int = 0) -> None:
        """The persistent entry over ``[base, base + count)``; the pointers are
        device addresses (0 for an optional one left out)."""
        vp = lambda v: ctypes.c_void_p(int(v) or None)   # noqa: E731
        check(lib().hkb_entry_launch_persist(self._h, block._h, int(base), int(count), int(n_samples),
                                             vp(next_ptr), vp(util), vp(steps), vp(stepsum), int(chunk),
                                             int(grid), vp(stream)),
              f"launching {self.name!r}")

    def launch_range(self, block: "ArgBlock", base: int, count: int, n_samples: int, steps: int = 0,
                     stepsum: int = 0, stream: int = 0) -> None:
        """The contiguous-range entry over ``[base, base + count)``; ``steps``
        and ``stepsum`` are device addresses (0 when not reported)."""
        vp = lambda v: ctypes.c_void_p(int(v) or None)   # noqa: E731
        check(lib().hkb_entry_launch_range(self._h, block._h, int(base), int(count), int(n_samples),
                                           vp(steps), vp(stepsum), vp(stream)),
              f"launching {self.name!r}")


class ArgBlock:
    """``hawk._core.ArgBlock``'s device twin: one by-value cell per slot."""

    def __init__(self, kinds) -> None:
        self.kinds = list(kinds)
        arr = (ctypes.c_char_p * len(self.kinds))(*[k.encode() for k in self.kinds])
        self._h = ctypes.c_void_p()
        check(lib().hkb_argblock_create(arr, len(self.kinds), ctypes.byref(self._h)), "hkb_argblock_create")

    def bind(self, slot: int, ptr: int, samples: int, stride: int = 1, device_type: int = 2,
             device_id: int = 0) -> None:
        check(lib().hkb_argblock_bind(self._h, int(slot), int(ptr), int(samples), int(stride),
                                      int(device_type), int(device_id)), f"binding slot {slot}")

    def rebind(self, slots, ptrs) -> None:
        n = len(slots)
        s = (ctypes.c_int64 * n)(*[int(x) for x in slots])
        p = (ctypes.c_int64 * n)(*[int(x) for x in ptrs])
        check(lib().hkb_argblock_rebind(self._h, s, p, n), "hkb_argblock_rebind")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and h.value and _LIB is not None:
            _LIB.hkb_argblock_free(h)
            self._h = None


def _ptr_array(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p) or None) for p in ptrs])


def cells_scratch_bytes(dtype: str, ncols: int, rows: int) -> int:
    return int(lib().hkb_cells_scratch_bytes(DTYPE[dtype], int(ncols), int(rows)))


def cells_finish(op: str, dtype: str, hi, comp, rows: int, scratch: int, out: int, stream: int = 0) -> None:
    """Rows of ``len(hi)`` columns finished into ``out`` (device pointers)."""
    check(lib().hkb_cells_finish(OP[op], DTYPE[dtype], len(hi), _ptr_array(hi),
                                 _ptr_array(comp) if comp is not None else None, int(rows),
                                 ctypes.c_void_p(int(scratch)), ctypes.c_void_p(int(out)),
                                 ctypes.c_void_p(int(stream) or None)), "hkb_cells_finish")


def cells_finish_noalloc(op: str, dtype: str, hi, comp, rows: int, out: int, stream: int = 0) -> None:
    """``cells_finish`` with the leaf partials in the library's static device
    array: for callers that cannot allocate device memory at finish time.  At
    most ``NOALLOC_LEAF_CAP`` leaf partials (all columns together) per call;
    calls that can overlap on the GPU share the array and race."""
    check(lib().hkb_cells_finish_noalloc(OP[op], DTYPE[dtype], len(hi), _ptr_array(hi),
                                         _ptr_array(comp) if comp is not None else None, int(rows),
                                         ctypes.c_void_p(int(out)), ctypes.c_void_p(int(stream) or None)),
          "hkb_cells_finish_noalloc")


NOALLOC_LEAF_CAP = 8192


def cells_leaves(op: str, dtype: str, hi, comp, rows: int, leaf_hi: int, leaf_comp: int, stream: int = 0) -> None:
    check(lib().hkb_cells_leaves(OP[op], DTYPE[dtype], len(hi), _ptr_array(hi),
                                 _ptr_array(comp) if comp is not None else None, int(rows),
                                 ctypes.c_void_p(int(leaf_hi)), ctypes.c_void_p(int(leaf_comp)),
                                 ctypes.c_void_p(int(stream) or None)), "hkb_cells_leaves")


def cells_tree(op: str, dtype: str, ncols: int, leaf_hi: int, leaf_comp: int, leaves: int, out: int,
               stream: int = 0) -> None:
    check(lib().hkb_cells_tree(OP[op], DTYPE[dtype], int(ncols), ctypes.c_void_p(int(leaf_hi)),
                               ctypes.c_void_p(int(leaf_comp)), int(leaves), ctypes.c_void_p(int(out)),
                               ctypes.c_void_p(int(stream) or None)), "hkb_cells_tree")


def cells_tree_ex(op: str, dtype: str, ncols: int, hi: int, comp: int, count: int, elem_stride: int,
                  col_stride: int, out: int, out_comp: int = 0, stream: int = 0) -> None:
    """The pairwise levels over strided partials; the root's (hi, comp) pair into
    ``out`` / ``out_comp`` when ``out_comp`` is given, else hi + comp into ``out``."""
    vp = lambda v: ctypes.c_void_p(int(v) or None)   # noqa: E731
    check(lib().hkb_cells_tree_ex(OP[op], DTYPE[dtype], int(ncols), vp(hi), vp(comp), int(count),
                                  int(elem_stride), int(col_stride), vp(out), vp(out_comp), vp(stream)),
          "hkb_cells_tree_ex")


class PeerArea:
    """This rank's exchange area for the peer-memory finish (``hkb_peer_*``):
    made on ``device``, its CUDA IPC handle in ``handle`` (bytes) until
    ``connect`` opens the other ranks' handles."""

    def __init__(self, device: int, rank: int, world: int, dtype: str, ncols: int) -> None:
        self._h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
        check(lib().hkb_peer_create(int(device), int(rank), int(world), DTYPE[dtype], int(ncols),
                                    ctypes.byref(self._h), buf), "hkb_peer_create")
        self.handle = buf.raw
        self.world = world

    def connect(self, handles: list) -> None:
        joined = b"".join(bytes(h) for h in handles)
        if len(joined) != self.world * PEER_HANDLE_BYTES:
            raise HawkError(f"hkb_peer_connect: {len(handles)} handles for a world of {self.world}")
        buf = ctypes.create_string_buffer(joined, len(joined))
        check(lib().hkb_peer_connect(self._h, buf), "hkb_peer_connect")

    def finish(self, op: str, leaf_hi: int, leaf_comp: int, leaves: int, out: int, seq: int,
               timeout_ns: int = 0, stream: int = 0) -> None:
        vp = lambda v: ctypes.c_void_p(int(v) or None)   # noqa: E731
        check(lib().hkb_peer_finish(self._h, OP[op], vp(leaf_hi), vp(leaf_comp), int(leaves), vp(out), int(seq),
                                    int(timeout_ns), vp(stream)), "hkb_peer_finish")

    def status(self) -> int:
        flags = ctypes.c_uint(0)
        check(lib().hkb_peer_status(self._h, ctypes.byref(flags)), "hkb_peer_status")
        return int(flags.value)

    def free(self) -> None:
        h = getattr(self, "_h", None)
        if h and h.value and _LIB is not None:
            _LIB.hkb_peer_free(h)
            self._h = None
