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
