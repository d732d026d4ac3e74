"""The device library's sin/cos against glibc's, on the CPU.

hk/math.cuh restates glibc's dbl-64 sin/cos (the reference host target's libm,
which its tests pin bit for bit: tests/test_math_parity.py:4-14) as compiled
for a host with FMA.  Its functions are ``__host__ __device__``, so the same
source text is compiled here with g++ and compared with this host's glibc on
1.6 million arguments over every range of the method: every bit must agree.
The GPU test ``test_trig_has_glibcs_bits`` checks the device compile of the
same text.

glibc picks its FMA build on hosts whose CPU has FMA and AVX2; elsewhere it
runs a build without FMA, whose results differ in about 0.1 % of arguments,
and this test is skipped.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from conftest import REPO

SOURCE = REPO / "tests" / "native" / "sincos_libm_check.cpp"
INCLUDE = REPO / "hawk_b200" / "csrc" / "include"


def host_has_fma() -> bool:
    try:
        flags = next(ln for ln in Path("/proc/cpuinfo").read_text().splitlines() if ln.startswith("flags"))
    except (OSError, StopIteration):
        return False
    words = set(flags.split())
    return "fma" in words and "avx2" in words


@pytest.mark.skipif(not host_has_fma(), reason="glibc runs its build without FMA on this CPU")
@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_device_sincos_source_has_glibcs_bits(tmp_path):
    exe = tmp_path / "sincos_libm_check"
    build = subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", f"-I{INCLUDE}", str(SOURCE),
                            "-o", str(exe), "-lm"], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe), "200000"], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "mismatches 0 of" in run.stdout
