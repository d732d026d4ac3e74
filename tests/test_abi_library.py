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
