"""The C-ABI library: it loads without a GPU and exports what its header declares."""

from __future__ import annotations

import ctypes
import re

from conftest import REPO

from hawk_b200 import abi


def declared_symbols() -> set:
    text = (REPO / "include" / "hawk_b200.h").read_text()
    return set(re.findall(r"^\s*(?:const char\*|int|void|size_t)\s+(hkb_\w+)\s*\(", text, re.M))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(abi.LIBRARY_PATH))
    names = declared_symbols()
    assert len(names) >= 18
    for name in names:
        assert hasattr(lib, name), name
    assert names == set(abi.SIGNATURES), "the ctypes binding covers exactly the header"


def test_layout_sizes_are_the_reference_mirror_sizes():
    # hawk/_contracts.py:58-92: GRefMirror 40, ScalarHandle 32, IntHandle 32, index 8, triple 24
    assert abi.layout_sizes() == [40, 32, 32, 8, 24]


def test_build_digest_is_stamped():
    d = abi.build_digest()
    assert re.fullmatch(r"[0-9a-f]{64}", d), d


def test_argblock_validates_kinds_and_slots():
    block = abi.ArgBlock(["gref", "handle", "f64", "nsamples"])
    value = ctypes.c_double(2.5)
    block.bind(2, ctypes.addressof(value), 1)
    block.bind(0, 0x1000, 64)
    import pytest
    from hawk_b200.errors import HawkError
    with pytest.raises(HawkError, match="outside"):
        block.bind(7, 0x1000, 1)
    with pytest.raises(HawkError, match="by-value"):
        block.rebind([2], [0x2000])
    with pytest.raises(HawkError, match="unknown descriptor kind"):
        abi.ArgBlock(["gref", "tensor"])


def test_cells_scratch_size():
    # two partials (hi, comp) per leaf of 4096 rows, per column
    assert abi.cells_scratch_bytes("float64", 3, 4096 * 5 + 1) == 2 * 3 * 6 * 8
    assert abi.cells_scratch_bytes("float32", 1, 1) == 2 * 4


def test_a_library_built_from_other_sources_is_refused():
    """The reference refuses a stale extension at import (hawk/__init__.py:128-209);
    the loader compares the digest the library was stamped with against its
    sources beside the package."""
    import pytest
    from hawk_b200.errors import HawkError

    assert abi.build_digest() == abi.sources_digest()
    abi.check_build_digest("a" * 64, None)               # no sources shipped: nothing to compare
    abi.check_build_digest("a" * 64, "a" * 64)
    with pytest.raises(HawkError, match="is stale: it was built from sources whose digest is aaaaaaaa"):
        abi.check_build_digest("a" * 64, "b" * 64)


def test_an_artifact_whose_unit_changed_is_refused_before_loading(tmp_path):
    """A sidecar records its unit's digest; a unit edited (or re-rendered)
    without its sidecar and CUBIN is refused by name, before the CUBIN is read."""
    import shutil

    import pytest
    from hawk_b200 import runtime
    from hawk_b200.errors import HawkError

    bundles = REPO / "hawk_b200" / "bundles"
    for suffix in (".cu", ".json"):
        shutil.copy(bundles / f"energy.float64{suffix}", tmp_path / f"energy.float64{suffix}")
    unit = tmp_path / "energy.float64.cu"
    unit.write_text(unit.read_text().replace("0.5", "0.25", 1))
    with pytest.raises(HawkError, match="energy.float64.cu is stale against its sidecar"):
        runtime.DeviceKernel(tmp_path, "energy", "float64", device=0)


def test_the_static_scratch_cap_is_the_headers():
    """The Python binding's cap of the allocation-free finish is the header's
    HKB_NOALLOC_LEAF_CAP (the refusal test sizes its case from it)."""
    text = (REPO / "include" / "hawk_b200.h").read_text()
    (cap,) = re.findall(r"#define\s+HKB_NOALLOC_LEAF_CAP\s+(\d+)", text)
    assert abi.NOALLOC_LEAF_CAP == int(cap)
    (rows,) = re.findall(r"#define\s+HKB_LEAF_ROWS\s+(\d+)", text)
    assert abi.LEAF_ROWS == int(rows)


def test_the_peer_finish_constants_are_the_headers_and_bad_shapes_are_refused():
    """The binding's handle size, rank limit and timeout bit are the header's;
    hkb_peer_create refuses a world or column count outside its area before it
    touches a device, and hkb_peer_finish a null area."""
    text = (REPO / "include" / "hawk_b200.h").read_text()
    for name, value in (("HKB_PEER_HANDLE_BYTES", abi.PEER_HANDLE_BYTES), ("HKB_PEER_MAX_RANKS", abi.PEER_MAX_RANKS),
                        ("HKB_PEER_TIMEOUT", abi.PEER_TIMEOUT)):
        (got,) = re.findall(rf"#define\s+{name}\s+(\d+)u?", text)
        assert value == int(got), name
    lib = abi.lib()
    out = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(abi.PEER_HANDLE_BYTES)
    assert lib.hkb_peer_create(0, 0, abi.PEER_MAX_RANKS + 1, 0, 3, ctypes.byref(out), handle) == 5
    assert "1..8 ranks" in lib.hkb_last_error().decode()
    assert lib.hkb_peer_create(0, 2, 2, 0, 3, ctypes.byref(out), handle) == 5
    assert lib.hkb_peer_create(0, 0, 2, 0, 9, ctypes.byref(out), handle) == 5
    assert out.value is None
    assert lib.hkb_peer_finish(None, 0, None, None, 1, None, 1, 0, None) == 1


def test_wait_errors_name_what_ran_out_and_a_drain_stops_the_unit():
    """The bits of a unit's error word (hk/stage.cuh kErrFullWait, kErrEmptyWait,
    kErrDrain) as the runtime reports them; a drain that ran out is fatal to
    the unit (later launches are refused)."""
    import pytest
    from types import SimpleNamespace

    from hawk_b200 import runtime
    from hawk_b200.errors import HawkError

    stage = (REPO / "hawk_b200" / "csrc" / "include" / "hk" / "stage.cuh").read_text()
    for name, bit in (("kErrFullWait", runtime.WAIT_FULL), ("kErrEmptyWait", runtime.WAIT_EMPTY),
                      ("kErrDrain", runtime.WAIT_DRAIN)):
        assert re.search(rf"{name} = {bit}u;", stage), name
    words = iter([runtime.WAIT_FULL, 0, runtime.WAIT_DRAIN])
    fake = SimpleNamespace(name="staged", poisoned="", library=SimpleNamespace(errors=lambda clear=True: next(words)))
    with pytest.raises(HawkError, match="did not arrive within the wait limit; the launch's outputs are incomplete"):
        runtime.DeviceKernel.check_waits(fake)
    runtime.DeviceKernel.check_waits(fake)
    with pytest.raises(HawkError, match="still in flight; the unit is not launched again"):
        runtime.DeviceKernel.check_waits(fake)
    assert fake.poisoned
