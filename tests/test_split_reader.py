"""The split build's reader-stage recogniser (no GPU).

A per-lane stage after a team stage whose body only copies scratch slices
(and single elements) into the kernel's outputs is emitted as a tiled copy
(``split._reader_copies`` / ``_reader_entry``); any other body keeps the lane
frame.  The committed team units re-render byte for byte
(``tests/test_target_row.py``); here the recogniser's refusals.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest

try:
    from hawk_b200 import configs  # noqa: F401  (brings up the reference front end)
    from hawk_b200.target import split
except Exception as exc:                                   # noqa: BLE001
    pytest.skip(f"the reference front end is not importable here ({exc})", allow_module_level=True)

from hawk.types import TensorType  # noqa: E402

SLICE = ("        const hk::Slice<Real, 4, 4> hawk_la0{lut_tm0_a.data() + "
         "static_cast<std::size_t>(static_cast<Int>(hawk_i)) * 16};")
ALIAS = "        const auto t2 = hawk_la0;"
STORE = "        mut_L[i] = t2;"
SCALAR = ("        mut_info[i] = lut_tm0_info[hk::SampleIndex::make(static_cast<std::size_t>("
          "static_cast<Int>(hawk_i)))].eval();")


def walk():
    types = {("mutable", "L"): TensorType((4, 4), "f64"), ("mutable", "info"): TensorType((), "i32"),
             ("lookup", "tm0_a"): TensorType((), "f64"), ("lookup", "tm0_info"): TensorType((), "i32")}
    return SimpleNamespace(arg_spec=tuple(types), slot_types=types)


def unit(*lines):
    return SimpleNamespace(body="\n".join(lines), sums=())


def test_a_copy_only_body_is_a_reader():
    assert split._reader_copies(unit(SLICE, ALIAS, STORE, SCALAR), walk()) == [
        ("mut_L", "lut_tm0_a", 16), ("mut_info", "lut_tm0_info", 1)]


@pytest.mark.parametrize("extra", ["        mut_L[i] = t2 * 2.0;", "        const auto t3 = t2;",
                                   "        hawk_acc += 1;"], ids=["scaled", "alias of alias", "other"])
def test_any_other_line_keeps_the_lane_frame(extra):
    assert split._reader_copies(unit(SLICE, ALIAS, STORE, extra), walk()) is None


def test_a_slice_whose_size_is_not_the_outputs_is_refused():
    wrong = SLICE.replace("* 16}", "* 15}")
    assert split._reader_copies(unit(wrong, ALIAS, STORE), walk()) is None
