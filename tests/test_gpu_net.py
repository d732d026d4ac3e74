"""The named net axis on the B200: K small models in one launch.

Lanes are (net, sample) of a ``Grid["net", "sample":S]``; each net's weights
are a row of a ``Table["net", "p":24]`` read at the lane's net; the loss keeps
the net label (``hawk.sum(..., over="sample")``) and its gradient wrt the
table is a keyed accumulate into it (the reference's tests/test_net_axis.py).
By default the loss's per-net sum and the gradient's table adds are atomic
commits; under ``policy="ordered"`` the loss runs as the block-sum stages and
the gradient as a per-lane log folded per net in lane order by a team stage
-- the same bits on every launch.  Values are held to the oracle (the
reference's loop over the nets, pinned by tests/golden/net.npz) at the
reference's tolerances: the device's tanh is not numpy's, so the bound is
relative, not bitwise.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from conftest import REPO  # noqa: E402
from hawk_b200 import runtime  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"
P, H = 24, 8
WIDTHS = (8, 3, 5, 1, 6)
EPS = np.finfo(np.float64).eps


def problem(k, s, seed=3):
    rng = np.random.default_rng(seed)
    w = rng.normal(size=(k, P)) * 0.7
    x, y = rng.normal(size=(k, s)), rng.normal(size=(k, s))
    wide = np.resize(np.asarray(WIDTHS), k)
    return w, x, y, (np.arange(H)[None, :] < wide[:, None]).astype(np.float64)


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a).ravel(), device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def loss_of(w, x, y, mask, ordered):
    k, s = x.shape
    name = f"net_loss_{s}" + ("_ordered" if ordered else "")
    out = torch.full((k,), float("nan"), dtype=torch.float64, device="cuda")
    if not ordered:
        out.zero_()                     # the default loss adds its commits into the plane
    runtime.run(runtime.load(BUNDLES, name), W=dev(w), mask=dev(mask), x=dev(x), y=dev(y), out=out)
    return host(out)


def grad_of(w, x, y, mask, ordered):
    k, s = x.shape
    name = f"net_grad_{s}" + ("_ordered" if ordered else "")
    bar_w = torch.zeros(k * P, dtype=torch.float64, device="cuda")
    if ordered:
        bar_w.fill_(float("nan"))       # the ordered fold stores every cell
    runtime.run(runtime.load(BUNDLES, name), W=dev(w), mask=dev(mask), x=dev(x), y=dev(y),
                bar_out=dev(np.ones(k)), bar_W=bar_w)
    return host(bar_w).reshape(k, P)


@pytest.mark.parametrize("ordered", [False, True])
def test_values_and_gradients_equal_the_loop_over_nets(golden, ordered):
    g = golden("net")
    w, x, y, mask = g["w_40"], g["x_40"], g["y_40"], g["mask_40"]
    np.testing.assert_allclose(loss_of(w, x, y, mask, ordered), g["loss_40"], rtol=1e-12)
    grad = grad_of(w, x, y, mask, ordered)
    np.testing.assert_allclose(grad, g["grad_40"], rtol=1e-11, atol=1e-11)
    dead = np.repeat(mask == 0.0, 3, axis=1)
    assert dead.any() and (grad[dead] == 0.0).all() and (grad[~dead] != 0.0).all()


@pytest.mark.parametrize("s", [40, 48])
def test_sixteen_thousand_nets_ordered_replay_bitwise_and_equal_the_loop(s):
    """16384 nets: three launches of the ordered loss and gradient, one set of
    bits each; equal to the loop on 256 of them; within the sum bound of the
    default (atomic) forms where those are built (S = 40)."""
    k = 16384
    w, x, y, mask = problem(k, s)
    losses = [loss_of(w, x, y, mask, True) for _ in range(3)]
    grads = [grad_of(w, x, y, mask, True) for _ in range(3)]
    assert losses[0].tobytes() == losses[1].tobytes() == losses[2].tobytes()
    assert grads[0].tobytes() == grads[1].tobytes() == grads[2].tobytes()
    want_loss, want_grad = oracle.net_axis(w, x, y, mask)
    np.testing.assert_allclose(losses[0], want_loss, rtol=1e-12)
    pick = np.random.default_rng(1).choice(k, 256, replace=False)
    np.testing.assert_allclose(grads[0][pick], want_grad[pick], rtol=1e-10, atol=1e-10)
    if s == 40:
        comp = loss_of(w, x, y, mask, False)
        np.testing.assert_allclose(losses[0], comp, rtol=8 * s * EPS)
        cg = grad_of(w, x, y, mask, False)
        np.testing.assert_allclose(grads[0], cg, rtol=1e-9, atol=1e-9 * np.abs(cg).max())


def test_perturbing_one_net_moves_no_other_net():
    w, x, y, mask = problem(5, 40)
    base = loss_of(w, x, y, mask, True), grad_of(w, x, y, mask, True)
    w2, x2, y2 = w.copy(), x.copy(), y.copy()
    w2[2] += 0.5
    x2[2] *= 1.5
    y2[2] -= 1.0
    moved = loss_of(w2, x2, y2, mask, True), grad_of(w2, x2, y2, mask, True)
    keep = [0, 1, 3, 4]
    assert np.array_equal(moved[0][keep], base[0][keep])
    assert np.array_equal(moved[1][keep], base[1][keep])
    assert not np.array_equal(moved[1][2], base[1][2])


def test_ordered_gradient_is_the_device_loss_slope():
    w, x, y, mask = problem(5, 40, seed=7)
    grad = grad_of(w, x, y, mask, True)
    rng = np.random.default_rng(2)
    for net, col in zip(rng.integers(0, 5, 8), rng.integers(0, P, 8)):
        up, dn = w.copy(), w.copy()
        up[net, col] += 1e-6
        dn[net, col] -= 1e-6
        slope = (loss_of(up, x, y, mask, True)[net] - loss_of(dn, x, y, mask, True)[net]) / 2e-6
        assert abs(grad[net, col] - slope) <= 1e-6 * max(1.0, abs(slope))


@pytest.mark.parametrize("ordered", [False, True])
def test_a_gradient_plane_smaller_than_its_table_is_refused(ordered):
    """bar_W takes adds at W's own indices: it must hold W's elements
    (hawk/_bind_checks.py:384-395)."""
    from hawk_b200.errors import HawkError

    w, x, y, mask = problem(5, 40)
    name = "net_grad_40" + ("_ordered" if ordered else "")
    with pytest.raises(HawkError, match=r"the gradient of the lookup plane 'W' \(shape \(120,\)\) needs"):
        runtime.run(runtime.load(BUNDLES, name), W=dev(w), mask=dev(mask), x=dev(x), y=dev(y),
                    bar_out=dev(np.ones(5)), bar_W=torch.zeros(119, dtype=torch.float64, device="cuda"))
