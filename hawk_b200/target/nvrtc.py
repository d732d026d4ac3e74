"""NVRTC compile of a b200 unit, pinned to sm_100a.

The reference compiles its device unit with NVRTC at the running GPU's arch,
or PTX at the toolkit maximum when that GPU is newer (hawk/compile/nvrtc.py:479-507,
hawk/compile/toolchain.py:240-305).  The b200 target has one arch: every unit
is compiled to an sm_100a CUBIN (SASS, no PTX JIT at load), with

* ``-std=c++17``, ``-default-device`` (a lambda in the body is device code) and the device library's include root, nothing else on the
  include path (NVRTC carries no standard headers; the library needs none);
* ``--fmad=false``: the body's multiplies and adds are not contracted into
  FMAs, so each rounds exactly as the reference's host build does
  (``-ffp-contract=off``, hawk/compile/toolchain.py:897-900).  The device
  library's own double-double arithmetic calls FMA explicitly;
* ``-lineinfo`` for profiler source attribution, and ``-Xptxas -v`` whose
  register/spill report is kept in the sidecar (as the reference's ``ptxas``
  block, hawk/artifact/sidecar.py:400-403).

This module has no dependency on the reference's front end: a runtime that
holds only a unit's text can compile it here.
"""

from __future__ import annotations

import re
from pathlib import Path

from ..errors import HawkError

ARCH = "sm_100a"
#: The device library's include root (``#include "hk/hawk_b200.cuh"``).
INCLUDE_DIR = Path(__file__).resolve().parent.parent / "csrc" / "include"


def options(extra=()) -> list:
    return [f"-arch={ARCH}", "-std=c++17", "-default-device", "--fmad=false", "-lineinfo",
            "-Xptxas", "-v", f"-I{INCLUDE_DIR}", *extra]


def _check(result, what: str) -> None:
    err = result[0] if isinstance(result, tuple) else result
    if int(err) != 0:
        raise HawkError(f"NVRTC {what} failed: {err!r}")


def compile_cubin(text: str, name: str, extra=()) -> tuple:
    """``(cubin bytes, log, ptxas)`` for one unit; a failed compile raises
    ``HawkError`` carrying NVRTC's log."""
    try:
        from cuda.bindings import nvrtc
    except ImportError as exc:          # the product path needs the compiler; no fallback
        raise HawkError("the b200 target compiles with NVRTC (cuda-python's cuda.bindings.nvrtc), "
                        "which is not importable here") from exc
    err, prog = nvrtc.nvrtcCreateProgram(text.encode(), f"{name}.cu".encode(), 0, [], [])
    _check(err, "program creation")
    opts = [o.encode() for o in options(extra)]
    try:
        res = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
        err, size = nvrtc.nvrtcGetProgramLogSize(prog)
        log_buf = b" " * size
        nvrtc.nvrtcGetProgramLog(prog, log_buf)
        log = log_buf.decode(errors="replace").rstrip("\x00 \n")
        if int(res[0]) != 0:
            raise HawkError(f"NVRTC could not compile {name!r} for {ARCH}:\n{log}")
        err, size = nvrtc.nvrtcGetCUBINSize(prog)
        _check(err, "CUBIN size")
        cubin = b" " * size
        _check(nvrtc.nvrtcGetCUBIN(prog, cubin), "CUBIN fetch")
    finally:
        nvrtc.nvrtcDestroyProgram(prog)
    return cubin, log, ptxas_report(log)


_PTXAS = re.compile(r"Function properties for (\w+)|Used (\d+) registers|(\d+) bytes stack frame, "
                    r"(\d+) bytes spill stores, (\d+) bytes spill loads")


def ptxas_report(log: str) -> dict:
    """``{entry: {regs, stack_B, spill_store_B, spill_load_B}}`` from the ptxas report."""
    out: dict = {}
    current = None
    for line in log.splitlines():
        m = re.search(r"Compiling entry function '(\w+)'", line) or re.search(r"Function properties for (\w+)", line)
        if m:
            current = m.group(1)
            out.setdefault(current, {})
            continue
        if current is None:
            continue
        m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m:
            out[current].update(stack_B=int(m.group(1)), spill_store_B=int(m.group(2)),
                                spill_load_B=int(m.group(3)))
        m = re.search(r"Used (\d+) registers", line)
        if m:
            out[current]["regs"] = int(m.group(1))
    return out
