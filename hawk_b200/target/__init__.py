"""The b200 target: a row for the reference's targets table, and the bundle build.

A target is one row of ``hawk.targets.TARGETS`` (hawk/targets/__init__.py:37-71;
docs/content/contributing/add_a_target.md:3-75): a writer, a wrapper, a
toolchain, how the kernel is entered, the artifact format and suffixes.  The
b200 row pairs the b200 writer (the reference's aether spelling over the
hand-written ``hk`` device library) with the b200 wrapper, compiles with NVRTC
at sm_100a only, and produces a CUBIN entered as a device kernel.

``install()`` adds the row to the reference's table, so the reference's own
``hawk.build(..., targets=("b200",))`` renders a b200 unit through the same
seams as its ``cuda`` row.  The reference's compile step forks on the row's
toolchain in one function (hawk/compile/drivers.py:417) and knows two
toolchains; ``build()`` here is the b200 row's own render + NVRTC + sidecar
step, which a maintainer wires into that fork (the branch is shown in the
integration notes).  Everything in this package imports the reference's front
end and is used where it is importable; the runtime (``hawk_b200.runtime``)
never imports it.
"""

from __future__ import annotations

from .nvrtc import ARCH, compile_cubin

#: The toolchain word of the b200 row (a new value beside the reference's GPU/CPU).
NVRTC_SM100A = "nvrtc-sm100a"


def row():
    """The b200 ``Target`` row: its ``features`` are exactly the entries of the
    reference's feature table (hawk/targets/features.py:74-152) the b200 build
    makes (``BUILT_FEATURES``); the render refuses the rest by name."""
    from hawk.targets import Target
    from .assemble import BUILT_FEATURES
    from .wrapper import B200
    from .writer import B200_WRITER

    return Target("b200", "builds for the B200 (sm_100a) through NVRTC", B200_WRITER, B200,
                  NVRTC_SM100A, "device", "cubin", ".cubin", ".cu", BUILT_FEATURES)


def install() -> None:
    """Add the b200 row to ``hawk.targets.TARGETS`` (idempotent)."""
    from hawk.targets import TARGETS

    TARGETS["b200"] = row()


def __getattr__(name):
    if name in ("render_unit", "Unit"):
        from . import assemble
        return getattr(assemble, name)
    if name in ("build", "build_kernel"):
        from . import build as _build
        return getattr(_build, name)
    raise AttributeError(name)


__all__ = ["ARCH", "NVRTC_SM100A", "compile_cubin", "install", "row"]
