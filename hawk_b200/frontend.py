"""Bring up the reference's front end (trace, IR, autodiff, renderer) for a build.

hawk's front end is used unchanged to trace kernels, derive their VJP/JVP and
render bodies.  Importing it needs two modules the reference gets from its own
native build and a third-party package:

* ``hawk._core`` -- the reference's nanobind extension (src/hawk_core.cpp).
  The package's import-time self-check (hawk/__init__.py:130-209) reads its
  ``build_digest()`` and ``layout_sizes()``.  The stand-in here answers the
  digest by the reference's own rule (sha256 over ``src/*`` and
  ``CMakeLists.txt`` beside the package, hawk/__init__.py:128-141) and the
  layout sizes from this build's C-ABI library when it is built (else the
  mirror sizes the device library asserts, 40/32/32/8/24).  Its host-execution
  classes (``HostLibrary``, ``ArgBlock``) refuse: the b200 path runs on the
  device through ``hawk_b200.runtime``.
* ``aether_dsc`` -- the reference's numerics payload package, used only by its
  own device/host compiles and the embedded C export; a stub that refuses
  when used.

The front end is found on ``sys.path``, else under the directory named by
``HAWK_FRONTEND``, else in a checkout named ``reference`` beside this
repository.  Only the build side imports this module.
"""

from __future__ import annotations

import hashlib
import importlib
import importlib.util
import os
import sys
import types
from pathlib import Path

from .errors import HawkError

#: Where the front end is looked for last: a checkout named ``reference``
#: beside this repository.
_FALLBACK_ROOTS = (str(Path(__file__).resolve().parents[2] / "reference"),)


def _root_of(candidate) -> Path | None:
    if not candidate:
        return None
    p = Path(candidate)
    return p if (p / "hawk" / "__init__.py").is_file() else None


def _source_digest(root: Path) -> str:
    files = [p for p in root.glob("src/*") if p.is_file()] + [root / "CMakeLists.txt"]
    stream = []
    for path in sorted(files, key=lambda p: p.relative_to(root).as_posix()):
        stream.append(f"{path.relative_to(root).as_posix()}\n{hashlib.sha256(path.read_bytes()).hexdigest()}\n")
    return hashlib.sha256("".join(stream).encode()).hexdigest()


def _layout_sizes() -> list:
    try:
        from . import abi
        return abi.layout_sizes()
    except Exception:                                   # noqa: BLE001 -- the library may be unbuilt
        return [40, 32, 32, 8, 24]


class _HostRefusal:
    """The reference's host-execution classes: not part of the b200 path."""

    def __init__(self, *args, **kwargs):
        raise HawkError("hawk._core host execution is not part of the b200 path; "
                        "load the artifact with hawk_b200.load and run it with hawk_b200.run")


def _core_module(root: Path) -> types.ModuleType:
    core = types.ModuleType("hawk._core")
    digest = _source_digest(root) if (root / "CMakeLists.txt").is_file() else ""
    core.build_digest = lambda: digest
    core.layout_sizes = _layout_sizes
    core.build_info = lambda: {"index_type_bytes": 8, "compiler": "b200-frontend"}

    def stat_many(paths):
        sizes, mtimes = [], []
        for p in paths:
            try:
                st = os.stat(p)
                sizes.append(st.st_size)
                mtimes.append(st.st_mtime_ns)
            except OSError:
                sizes.append(-1)
                mtimes.append(-1)
        return sizes, mtimes

    core.stat_many = stat_many
    core.ArgBlock = _HostRefusal
    core.HostLibrary = _HostRefusal
    return core


def _aether_stub() -> tuple:
    def refuse(*args, **kwargs):
        # The front end's own refusal type: its callers that can do without the
        # payload (the libc-name probe, hawk/compile/toolchain.py:752-783) catch it.
        from hawk.ir import HawkError as FrontEndError
        raise FrontEndError("aether_dsc (the reference's numerics payload) is not used on the b200 path")

    class _Refusing:
        def __init__(self, *a, **k):
            refuse()

    pkg = types.ModuleType("aether_dsc")
    c_core = types.ModuleType("aether_dsc.c_core")
    c_core.CORE_VERSION = "b200-stub"
    c_core.CFunction = _Refusing
    c_core.struct = refuse
    c_core.function = refuse
    c_core.emit = refuse
    pkg.c_core = c_core
    pkg.payload = refuse
    pkg.seal = refuse
    pkg.Payload = _Refusing
    return pkg, c_core


def load():
    """Import and return the reference's ``hawk`` package (idempotent)."""
    if "hawk" in sys.modules and getattr(sys.modules["hawk"], "kernel", None) is not None:
        return sys.modules["hawk"]
    root = None
    spec = importlib.util.find_spec("hawk") if "hawk" not in sys.modules else None
    if spec is not None and spec.origin:
        root = Path(spec.origin).resolve().parent.parent
    for candidate in (os.environ.get("HAWK_FRONTEND"), *_FALLBACK_ROOTS):
        if root is None:
            root = _root_of(candidate)
    if root is None:
        raise HawkError("the hawk front end is not importable: put it on sys.path or name its "
                        "checkout in HAWK_FRONTEND (only building bundles needs it)")
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    sys.modules.setdefault("hawk._core", _core_module(root))
    if "aether_dsc" not in sys.modules:
        pkg, c_core = _aether_stub()
        sys.modules["aether_dsc"] = pkg
        sys.modules["aether_dsc.c_core"] = c_core
    import hawk

    return hawk


def available() -> bool:
    """Whether the front end can be brought up here."""
    try:
        load()
        return True
    except Exception:                                   # noqa: BLE001
        return False
