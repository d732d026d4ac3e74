"""Host-side slot rules of the runtime (no GPU): which written plane is the
adjoint of a lookup plane, and so must hold that plane's elements."""

from __future__ import annotations


def test_the_adjoint_of_a_lookup_plane_is_named_by_its_prefix():
    """bar_<plane> of a lookup plane, accumulated or stored by a fold stage
    (hawk/ir/walk.py:144-152); a bar_ plane of a per-sample input is not one."""
    from hawk_b200.runtime import adjoint_like

    slots = [("accum_out", "bar_table"), ("lookup", "table"), ("per_sample", "x"), ("wide_out", "bar_W"),
             ("lookup", "W"), ("out", "bar_x")]
    assert adjoint_like(slots) == {"bar_table": "table", "bar_W": "W"}


def test_a_gradient_plane_smaller_than_its_table_is_named():
    from types import SimpleNamespace

    from hawk_b200.runtime import adjoint_errors

    planes = {"W": SimpleNamespace(size=120, shape=(120,)), "bar_W": SimpleNamespace(size=119, shape=(119,))}
    (msg,) = adjoint_errors({"bar_W": "W"}, planes)
    assert "the gradient of the lookup plane 'W' (shape (120,)) needs that many elements, got shape (119,)" in msg
    planes["bar_W"] = SimpleNamespace(size=120, shape=(120,))
    assert adjoint_errors({"bar_W": "W"}, planes) == []


def test_the_teams_a_stage_launches():
    """hawk/_lane_bind.py:123-134: lanes, keys x groups, an ordered scatter's
    target cells, and its chunks -- times the warps the b200 chunk stage walks
    each chunk with."""
    from types import SimpleNamespace

    from hawk_b200.runtime import SplitKernel

    fake = SimpleNamespace(scatter_chunks=SplitKernel.scatter_chunks, keyed_size=lambda keyed, n: n // 8)
    grid = lambda record, n, count, sizes: SplitKernel.grid(fake, record, n, count, sizes)  # noqa: E731
    assert grid({"grid": "lanes"}, 100, 37, {}) == 37
    assert grid({"grid": "keys", "keyed": {"width": 1}, "groups": 64}, 800, 800, {}) == 100 * 64
    assert grid({"grid": "targets", "of": "acc"}, 20000, 20000, {"acc": 7}) == 7
    assert grid({"grid": "chunks", "of": "acc", "groups": 8}, 20000, 20000, {"acc": 7}) == 256 * 8
    assert grid({"grid": "chunks", "of": "acc"}, 50, 50, {"acc": 200}) == 1
