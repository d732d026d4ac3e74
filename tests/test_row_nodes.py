"""The row-sum node arithmetic of the device library, on the CPU.

hk/sample_sum.cuh's node helpers are ``__host__ __device__``: the same source
text is compiled here with g++ and a 32-sample row tree built from them (the
device's order: first level by the residual alone, later nodes unchecked,
either operand first, the root settled by ``root_comp``) is compared bit for
bit with the reference's node rule -- the ordered Fast2Sum residual with + 0
and a finiteness test at every node (hawk/_cells.py:44-49) -- on rows drawn
to hit zero residuals, signed zeros, exact cancellations, overflow and NaN.
It also checks that the 2Sum residual is never -0 on every sign combination
of a set of special magnitudes (the reason the device adds no + 0).
"""

from __future__ import annotations

import shutil
import subprocess

import pytest

from conftest import REPO

SOURCE = REPO / "tests" / "native" / "row_nodes_check.cpp"
INCLUDE = REPO / "hawk_b200" / "csrc" / "include"


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_device_row_nodes_make_the_reference_rows(tmp_path):
    exe = tmp_path / "row_nodes_check"
    build = subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", f"-I{INCLUDE}", str(SOURCE),
                            "-o", str(exe)], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe), "200000"], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "mismatches 0 of 200000 rows" in run.stdout
