"""The symmetric eigenproblem on the B200: ``w, V, info = hawk.math.eigh(A)``
per sample (the one-thread form, n <= 32).

The device library's cyclic Jacobi (hk/linalg.cuh ``eigh``) is the order of
operations the reference restates in hawk/embedded/linalg.py:302-399, as is
the oracle's, so the device equals the oracle bit for bit -- eigenvalues,
eigenvectors, the status word (bit 2: two eigenvalues closer than the
tolerance) -- and the values-only build (no V accumulated) gives the same
eigenvalues.  The oracle is pinned against numpy's eigh through the reference
interpreter (tests/test_oracle_golden.py).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from hawk_b200 import runtime  # noqa: E402

BUNDLES = REPO / "hawk_b200" / "bundles"


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def symmetric(n, lanes, seed):
    rng = np.random.default_rng(seed)
    mats = []
    for lane in range(lanes):
        g = rng.standard_normal((n, n))
        a = (g + g.T) / 2 + (0.3 * rng.standard_normal((n, n)) if lane % 3 == 1 else 0.0)  # some not symmetric
        if lane % 7 == 2:                               # a repeated eigenvalue
            q, _ = np.linalg.qr(rng.standard_normal((n, n)))
            a = (q * np.r_[np.ones(n // 2), np.linspace(2, 3, n - n // 2)]) @ q.T
        mats.append(a)
    return np.ascontiguousarray(np.moveaxis(np.stack(mats), 0, -1))


@pytest.mark.parametrize("lanes", [1, 33, 1000])
def test_eigh_is_the_oracle_bit_for_bit(lanes):
    A = symmetric(6, lanes, lanes)
    w = torch.full((6, lanes), float("nan"), dtype=torch.float64, device="cuda")
    V = torch.full((6, 6, lanes), float("nan"), dtype=torch.float64, device="cuda")
    info = torch.full((lanes,), -7, dtype=torch.int32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "sym_eigen"), A=dev(A), w=w, V=V, info=info)
    want_w, want_V, want_info = oracle.sym_eigen(A)
    np.testing.assert_array_equal(host(info), want_info)
    np.testing.assert_array_equal(host(w), want_w)
    np.testing.assert_array_equal(host(V), want_V)
    np.testing.assert_allclose(host(w), want_w, rtol=1e-12, atol=0)
    if lanes > 2:
        assert host(info)[2] & 2


def test_eigenvalues_alone_match_the_full_solve():
    lanes = 500
    A = symmetric(4, lanes, 4)
    w = torch.full((4, lanes), float("nan"), dtype=torch.float64, device="cuda")
    info = torch.full((lanes,), -7, dtype=torch.int32, device="cuda")
    runtime.run(runtime.load(BUNDLES, "sym_eigvals"), A=dev(A), w=w, info=info)
    want_w, _V, want_info = oracle.sym_eigen(A)
    np.testing.assert_array_equal(host(w), want_w)
    np.testing.assert_array_equal(host(info), want_info)
