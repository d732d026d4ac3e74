"""The allocation-free cells finish against the finish that takes caller scratch.

``hkb_cells_finish_noalloc`` is for callers that cannot allocate device memory
when they finish a reduction (a framework that owns every device allocation and
hands its plugins only inputs and outputs, or a loop with a fixed memory budget).
It keeps the leaf partials in a static array of the library instead of caller
scratch.  Its cells must equal ``hkb_cells_finish``'s bit for bit, on two calls
in a row (the array keeps the previous call's contents, which must not leak into
the next), for both element types and the max/min ops; and a size beyond the
static array is refused before anything runs.

This file is collected last, so a run that stops at its first failure has run
every other test already; it also passes alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from hawk_b200 import abi  # noqa: E402
from hawk_b200.errors import HawkError  # noqa: E402


def _rows(rows: int, ncols: int, dtype: str, seed: int):
    rng = np.random.default_rng(seed)
    np_dt = np.float64 if dtype == "float64" else np.float32
    hi = rng.standard_normal((ncols, rows)) * np.exp(rng.uniform(-10, 10, (ncols, rows)))
    comp = rng.standard_normal((ncols, rows)) * np.abs(hi) * 1e-17
    return (torch.as_tensor(hi.astype(np_dt), device="cuda"), torch.as_tensor(comp.astype(np_dt), device="cuda"))


def _finish_both(op: str, dtype: str, rows: int, ncols: int, seed: int):
    hi, comp = _rows(rows, ncols, dtype, seed)
    tdt = torch.float64 if dtype == "float64" else torch.float32
    his = [hi[k].data_ptr() for k in range(ncols)]
    comps = [comp[k].data_ptr() for k in range(ncols)] if op == "sum" else None
    scratch = torch.empty(abi.cells_scratch_bytes(dtype, ncols, rows), dtype=torch.uint8, device="cuda")
    want = torch.full((ncols,), float("nan"), dtype=tdt, device="cuda")
    got = torch.full((ncols,), float("nan"), dtype=tdt, device="cuda")
    abi.cells_finish(op, dtype, his, comps, rows, scratch.data_ptr(), want.data_ptr())
    abi.cells_finish_noalloc(op, dtype, his, comps, rows, got.data_ptr())
    torch.cuda.synchronize()
    return got.cpu().numpy(), want.cpu().numpy()


@pytest.mark.parametrize("dtype", ["float64", "float32"])
def test_two_calls_in_a_row_equal_the_scratch_finish(dtype):
    # a large call, then a smaller one whose leaves sit where the first call's were
    for call, (rows, ncols, seed) in enumerate(((131077 * 3 + 11, 3, 1), (5000, 2, 2))):
        got, want = _finish_both("sum", dtype, rows, ncols, seed)
        assert np.isfinite(want).all()
        np.testing.assert_array_equal(got, want, err_msg=f"call {call}")


@pytest.mark.parametrize("op", ["max", "min"])
def test_extreme_ops_equal_the_scratch_finish(op):
    for seed in (3, 4):
        got, want = _finish_both(op, "float64", 70001, 3, seed)
        np.testing.assert_array_equal(got, want)


def test_a_size_beyond_the_static_scratch_is_refused():
    one = torch.zeros(1, dtype=torch.float64, device="cuda")
    ptrs = [one.data_ptr()] * 3
    leaves_each = abi.NOALLOC_LEAF_CAP // 3 + 1
    rows = leaves_each * abi.LEAF_ROWS
    out = torch.zeros(3, dtype=torch.float64, device="cuda")
    with pytest.raises(HawkError, match="static scratch"):
        abi.cells_finish_noalloc("sum", "float64", ptrs, ptrs, rows, out.data_ptr())


@pytest.mark.parametrize("dtype", ["float64", "float32"])
def test_a_call_at_exactly_the_cap_equals_the_scratch_finish(dtype):
    """ncols * leaves == HKB_NOALLOC_LEAF_CAP: every partial slot of the static
    array is used (for float64 the companions' half ends at its last byte), on
    two calls in a row."""
    ncols = 4
    rows = (abi.NOALLOC_LEAF_CAP // ncols) * abi.LEAF_ROWS
    for seed in (5, 6):
        got, want = _finish_both("sum", dtype, rows, ncols, seed)
        assert np.isfinite(want).all()
        np.testing.assert_array_equal(got, want)
