"""Build the native parts of hawk_b200 in-tree.

* ``hawk_b200/lib/libhawk_b200.so`` -- the C ABI of include/hawk_b200.h (the
  loader, argument blocks, launches and the finish-tree kernels), compiled by
  nvcc for sm_100a with the CUDA runtime linked statically (so it loads on a
  host without a GPU driver);
* the b200 bundles' CUBINs -- every ``hawk_b200/bundles/*.cu`` unit compiled by
  NVRTC for sm_100a (``hawk_b200.target.nvrtc``), beside its unit.

The library's build digest is the sha256 over its sources, stamped in at
compile time (``hkb_build_digest``), the rule the reference applies to its own
binding (hawk/__init__.py:128-141).

    python -m hawk_b200.csrc.build          # library + CUBINs
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
REPO = PKG.parent
LIB_DIR = PKG / "lib"
LIBRARY = LIB_DIR / "libhawk_b200.so"
SOURCES = [PKG / "csrc" / "shim" / "hawk_b200.cu"]
HEADERS = sorted((PKG / "csrc" / "include" / "hk").glob("*.cuh")) + [REPO / "include" / "hawk_b200.h"]
BUNDLES = PKG / "bundles"

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (Path(cand).exists() or cand == "nvcc"):
            return cand
    return "nvcc"


def source_digest() -> str:
    h = hashlib.sha256()
    for path in sorted(SOURCES + HEADERS):
        h.update(path.relative_to(REPO).as_posix().encode() + b"\n")
        h.update(hashlib.sha256(path.read_bytes()).hexdigest().encode() + b"\n")
    return h.hexdigest()


def build_library(force: bool = False) -> Path:
    """Compile libhawk_b200.so when a source is newer than it (or ``force``)."""
    LIB_DIR.mkdir(exist_ok=True)
    newest = max(p.stat().st_mtime for p in SOURCES + HEADERS)
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= newest:
        return LIBRARY
    cmd = [nvcc(), *NVCC_FLAGS, f"-DHKB_BUILD_DIGEST=\"{source_digest()}\"",
           f"-I{REPO / 'include'}", f"-I{PKG / 'csrc' / 'include'}",
           *map(str, SOURCES), "-o", str(LIBRARY)]
    run = subprocess.run(cmd, capture_output=True, text=True)
    if run.returncode != 0:
        raise RuntimeError(f"nvcc failed building {LIBRARY.name}:\n{run.stderr}")
    return LIBRARY


def build_cubins(force: bool = False) -> list:
    """NVRTC-compile every bundle unit whose CUBIN is missing or older than it
    (or than a device-library header)."""
    from hawk_b200.target.nvrtc import compile_cubin

    headers_mtime = max(p.stat().st_mtime for p in HEADERS)
    built = []
    for unit in sorted(BUNDLES.glob("*.cu")) + sorted((BUNDLES / "staged").glob("*.cu")):
        cubin = unit.with_suffix(".cubin")
        if (not force and cubin.exists()
                and cubin.stat().st_mtime >= max(unit.stat().st_mtime, headers_mtime)):
            continue
        entry = unit.name.split(".")[0]
        image, _log, _ptxas = compile_cubin(unit.read_text(), entry)
        cubin.write_bytes(image)
        built.append(cubin)
    return built


def main(argv=None) -> int:
    force = "--force" in (argv or sys.argv[1:])
    print(build_library(force))
    for c in build_cubins(force):
        print(c)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
