"""Test configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs on a host without a GPU: the oracle against the golden
vectors, the emitter (where the hawk front end is importable), the runtime's
host-side logic, the C-ABI library's exports, multi-rank logic over gloo.
``-m gpu`` runs the parity tests proper on a B200, through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); run with -m gpu")


def pytest_sessionstart(session):
    """Bring the in-tree builds up to date before any test loads them: the
    C-ABI library (nvcc) when a source or header is newer than it -- the loader
    refuses a library stale against its sources -- and each bundle's CUBIN
    (NVRTC) when its unit or a header is newer.  Each is a no-op when current;
    without a compiler the tests run on what is built."""
    try:
        from hawk_b200.csrc import build
        build.build_library()
        build.build_cubins()
    except Exception as exc:                     # noqa: BLE001 -- reported by the tests that need them
        print(f"conftest: the in-tree builds were not refreshed ({exc})")


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def load(name: str):
        if name not in cache:
            with np.load(GOLDEN / f"{name}.npz") as z:
                cache[name] = {k: z[k] for k in z.files}
        return cache[name]

    return load
