"""Planted faults the loader refuses by name, and device arrays bound through
the array interfaces (on the B200; nothing here launches a faulting kernel).

* A unit whose self-check exports are not this library's -- another
  ``eagle_abi_tag``, or mirror sizes it does not pack -- is refused at load,
  naming the field (src/hawk_core.cpp:366-389 of the reference; its tests
  plant the same faults, tests/test_serial_oracle.py:221).  The faulty unit is
  a committed unit with its exports line replaced, compiled by NVRTC here.
* A plane given as any object with ``__cuda_array_interface__`` (CuPy's and
  Numba's protocol) or ``__dlpack__`` binds like a torch tensor
  (hawk_b200/planes.py), with the same results.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

import oracle
from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from hawk_b200 import runtime, workloads  # noqa: E402
from hawk_b200.errors import HawkError  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"


def planted(directory, tag: str, sizes) -> None:
    """energy's unit with its exports replaced, compiled, beside a sidecar
    recording its digest."""
    from hawk_b200.target.nvrtc import compile_cubin

    text = (BUNDLES / "energy.float64.cu").read_text()
    assert text.count("HK_SELF_CHECK_EXPORTS") == 1
    exports = ('extern "C" __device__ unsigned int hk_error_flags = 0u;\n'
               f'extern "C" __device__ const char eagle_abi_tag[] = "{tag}";\n'
               'extern "C" __device__ unsigned long long eagle_layout_sizes[5] = {'
               + ", ".join(f"{s}ull" for s in sizes) + "};")
    text = text.replace("HK_SELF_CHECK_EXPORTS", exports)
    cubin, _log, _ptxas = compile_cubin(text, "energy")
    sidecar = json.loads((BUNDLES / "energy.float64.json").read_text())
    sidecar["b200"]["unit_digest"] = hashlib.sha256(text.encode()).hexdigest()
    (directory / "energy.float64.cu").write_text(text)
    (directory / "energy.float64.cubin").write_bytes(cubin)
    (directory / "energy.float64.json").write_text(json.dumps(sidecar))


def test_a_unit_of_another_abi_tag_is_refused_by_name(tmp_path):
    planted(tmp_path, "aether-abi/9", (40, 32, 32, 8, 24))
    with pytest.raises(HawkError, match="eagle_abi_tag is 'aether-abi/9', this library packs 'aether-abi/2'"):
        runtime.load(tmp_path, "energy")


def test_a_unit_of_other_mirror_sizes_is_refused_by_name(tmp_path):
    planted(tmp_path, "aether-abi/2", (40, 32, 32, 8, 16))
    with pytest.raises(HawkError, match=r"layout mismatch in sizeof\("):
        runtime.load(tmp_path, "energy")


def test_the_planted_unit_with_the_right_exports_loads_and_runs(tmp_path):
    """The control: the same replacement with this library's tag and sizes
    loads and gives the committed unit's bits."""
    planted(tmp_path, "aether-abi/2", (40, 32, 32, 8, 24))
    w = workloads.energy(1000, seed=3)
    out = torch.full((1000,), float("nan"), dtype=torch.float64, device="cuda")
    runtime.run(runtime.load(tmp_path, "energy"), v=torch.as_tensor(w["v"], device="cuda"), out=out)
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.energy(w["v"]))


class CudaArray:
    """Any device array exposing only ``__cuda_array_interface__`` (version 3)."""

    def __init__(self, t):
        self._t = t
        self.__cuda_array_interface__ = {
            "shape": tuple(t.shape), "typestr": {torch.float64: "<f8", torch.int32: "<i4"}[t.dtype],
            "data": (t.data_ptr(), False), "version": 3, "strides": None}


class DLPackArray:
    """Any device array exposing only ``__dlpack__`` / ``__dlpack_device__``."""

    def __init__(self, t):
        self._t = t

    def __dlpack__(self, *args, **kwargs):
        return self._t.__dlpack__(*args, **kwargs)

    def __dlpack_device__(self):
        return self._t.__dlpack_device__()


@pytest.mark.parametrize("wrap", [CudaArray, DLPackArray], ids=["cuda_array_interface", "dlpack"])
def test_array_interface_planes_bind_like_tensors(wrap):
    n = 4096 + 5
    w = workloads.gravity(n, seed=12)
    planes = {k: torch.as_tensor(w[k], device="cuda") for k in ("r1", "r2", "m1", "m2")}
    f, u = (torch.full(s, float("nan"), dtype=torch.float64, device="cuda") for s in ((3, n), (n,)))
    runtime.run(runtime.load(BUNDLES, "gravity"), **{k: wrap(v) for k, v in planes.items()}, G=w["G"],
                f=wrap(f), u=wrap(u))
    wf, wu = oracle.gravity(w["r1"], w["r2"], w["m1"], w["m2"], w["G"])
    np.testing.assert_array_equal(f.cpu().numpy(), wf)
    np.testing.assert_array_equal(u.cpu().numpy(), wu)


def test_a_read_only_array_interface_plane_is_refused_as_an_output():
    n = 100
    w = workloads.energy(n, seed=4)
    out = torch.zeros(n, dtype=torch.float64, device="cuda")
    ro = CudaArray(out)
    ro.__cuda_array_interface__["data"] = (out.data_ptr(), True)
    with pytest.raises(HawkError, match="out"):
        runtime.run(runtime.load(BUNDLES, "energy"), v=torch.as_tensor(w["v"], device="cuda"), out=ro)
