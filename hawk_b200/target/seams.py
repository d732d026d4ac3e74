"""The b200 row's two seams in the reference's build, and their wiring.

The reference builds a bundle for a list of targets in ``build_bundle``
(hawk/artifact/bundle.py:1349): per kernel it renders each row's translation
unit (``_sources`` -> ``render_source``, hawk/emit/wrapper.py:1132) and
compiles it through the one function that forks on the row's toolchain
(``compile_source``, hawk/compile/drivers.py:417); the artifacts, sidecars and
the manifest are then the reference's own.  A b200 row needs its own branch at
both seams:

* ``render_source`` -- the b200 unit (``render_unit``: the reference renderer's
  body in the device library's spelling inside the b200 entry and frames,
  the unit ``build_kernel`` would choose, register policy included) as the
  reference's ``Source``;
* ``compile_source`` -- NVRTC at sm_100a (``compile_cubin``), the CUBIN written
  into a content-addressed slot under the build's cache directory, returned as
  the reference's ``CompileResult`` with the ptxas report.

``wired()`` installs the b200 row and routes both seams for the b200 row
(every other row keeps the reference's own functions) for the duration of a
``with`` block: ``hawk.build([...], directory, targets=("b200",))`` then writes
b200 CUBINs, the reference's v2 sidecars and its manifest.  A maintainer adds
the two branches to the reference's functions instead (the integration
notes show them); the bodies are these.

Kernels the reference splits into stages (team-form linear algebra, sums read
back) are built by ``build_kernel`` / ``build_split_kernel``; the render seam
refuses them by name, as it refuses a segmented, active-set, thread-box or
fused-lane entry.
"""

from __future__ import annotations

import contextlib
import hashlib
import os
import tempfile
import threading
import time
from pathlib import Path
from types import SimpleNamespace

from ..errors import HawkError
from .nvrtc import compile_cubin, options

#: Compiles the render seam made while choosing the unit, by the unit text's
#: digest, so the compile seam does not compile the same text again; and the
#: chosen unit by (name, scalar mode), for the sidecar's b200 block.
_CHOSEN: dict = {}
_UNITS: dict = {}
_LOCK = threading.Lock()


def render_source(name, sinks, walk, target, *, mode=None, kind=None, exports: str = "", body=None, segment=None,
                  active=None, one_step=None, box=None, team=None, rows: int = 1):
    """The b200 branch of the reference's ``render_source``: the unit the b200
    row builds for the kernel, as the reference's ``Source``."""
    from hawk.emit.wrapper import Source

    from .build import choose_unit

    for label, value in (("segmented", segment), ("active-set", active), ("thread-box", box),
                         ("fused lane group", body), ("team", team)):
        if value is not None:
            raise HawkError(f"{name!r}: the {label} entry is not built through the b200 row's render seam")
    mode_id = getattr(mode, "id", None) or "float64"
    kernel = SimpleNamespace(name=name, sinks=sinks, walk=walk, one_step=one_step)
    unit, cubin, log, ptxas = choose_unit(kernel, name, mode_id)
    with _LOCK:
        _CHOSEN[hashlib.sha256(unit.text.encode()).hexdigest()] = (cubin, log, ptxas)
        _UNITS[(name, mode_id)] = (unit, ptxas)
    return Source(unit.text, unit.body, name, target.id, mode_id)


def sidecar_block(name: str, mode: str, walk, row) -> dict:
    """The ``b200`` block the reference's sidecar of a b200 artifact carries,
    naming the reference's artifact and source files (``<name>.cubin``,
    ``<name>.cu``)."""
    from .build import b200_block

    with _LOCK:
        unit, ptxas = _UNITS[(name, mode)]
    return json_safe(b200_block(unit, walk, ptxas, name, f"{name}{row.source}", f"{name}{row.artifact}"))


def json_safe(value):
    import json

    return json.loads(json.dumps(value, default=str))


def _cache_root(opts) -> Path:
    root = getattr(opts, "cache_dir", None) or os.environ.get("HAWK_CACHE_DIR")
    return Path(root) if root else Path(tempfile.gettempdir()) / "hawk_b200_cache"


def compile_source(source, name: str, opts, row):
    """The b200 branch of the reference's ``compile_source``: the unit compiled
    by NVRTC for sm_100a into ``<cache>/b200/<key>/<name>.cubin`` (the key: the
    unit text, the row, the scalar mode and the NVRTC options)."""
    from hawk.compile.drivers import CompileResult

    text = getattr(source, "text", source)
    argv = tuple(o for o in options() if not o.startswith("-I"))
    key = hashlib.sha256("\0".join([text, row.id, str(getattr(opts, "mode", "")), *argv]).encode()).hexdigest()
    slot = _cache_root(opts) / "b200" / key
    artifact, src = slot / f"{name}{row.artifact}", slot / f"{name}{row.source}"
    t0 = time.perf_counter()
    with _LOCK:
        chosen = _CHOSEN.get(hashlib.sha256(text.encode()).hexdigest())
    cubin, _log, ptxas = chosen if chosen is not None else compile_cubin(text, name)
    slot.mkdir(parents=True, exist_ok=True)
    src.write_text(text)
    artifact.write_bytes(cubin)
    return CompileResult(artifact, src, key, False, argv, time.perf_counter() - t0, (), ptxas)


@contextlib.contextmanager
def wired():
    """Within the block, the reference's build renders and compiles the b200
    row through the seams above (the row installed first)."""
    from unittest import mock

    import hawk.artifact.bundle as bundle
    import hawk.artifact.sidecar as sidecar
    import hawk.compile.drivers as drivers

    from . import install

    install()
    reference_render, reference_compile = bundle.render_source, drivers.compile_source
    reference_sidecar = bundle._sidecar

    def render(name, sinks, walk, target, **kw):
        if getattr(target, "id", None) == "b200":
            return render_source(name, sinks, walk, target, **kw)
        return reference_render(name, sinks, walk, target, **kw)

    def compile_(source, name, opts):
        from hawk.targets import TARGETS

        row = TARGETS.get(getattr(opts, "target", None))
        if row is not None and row.id == "b200":
            return compile_source(source, name, opts, row)
        return reference_compile(source, name, opts)

    def sidecar_of(kernel, *, name, smode, lead, **kw):
        meta = reference_sidecar(kernel, name=name, smode=smode, lead=lead, **kw)
        if lead == "b200":
            from hawk.targets import TARGETS

            meta["b200"] = sidecar_block(name, smode.id, kernel.walk, TARGETS["b200"])
        return meta

    # the sidecar records where a unit's third-party headers came from; a b200
    # unit includes only this build's device library
    with mock.patch.object(bundle, "render_source", render), mock.patch.object(bundle, "compile_source", compile_), \
            mock.patch.object(drivers, "compile_source", compile_), mock.patch.object(bundle, "_sidecar", sidecar_of), \
            mock.patch.object(sidecar, "_root_or_sealed_marker", lambda resolver: "hawk_b200/csrc/include"):
        yield
