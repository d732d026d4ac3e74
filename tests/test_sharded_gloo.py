"""The multi-GPU exchange, run as 2 CPU ranks over gloo.

Shards start on leaf boundaries, so every rank's leaf partials, gathered in
rank order, are the unsharded rows' leaves and the final tree is bit-identical
to one device's finish (hawk/_cells.py:94-119 over all rows).  The device
kernels are replaced by the oracle's two finish stages; what is tested is the
host logic: the shard cut, the gather and its ordering, uneven last shards.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hawk_b200 import sharded


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, queue):
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(77)
        x = rng.uniform(-2, 2, n)
        t = x + 0.1 * rng.standard_normal(n)
        bar_r = np.ones(n)
        hi_all, comp_all = oracle.poly_loss_vjp_rows(x, t, bar_r, 0.5, -1.0, 2.0)
        base, count = sharded.shard_range(n, world, rank)
        lo, hi = base // 32, -(-(base + count) // 32)
        leaves = sharded.leaves_of(count) if count else 0
        counts = [0] * world
        for r in range(world):
            counts[r] = sharded.leaves_of(sharded.shard_range(n, world, r)[1])
        width = max(counts)
        lh = np.zeros((3, width))
        lc = np.zeros((3, width))
        for k in range(3):
            if count:
                a, b = oracle.cells_leaves(hi_all[k, lo:hi], comp_all[k, lo:hi])
                lh[k, :leaves], lc[k, :leaves] = a, b
        g_hi, g_comp = sharded.gather_leaves(torch.from_numpy(lh), torch.from_numpy(lc), counts)
        got = [oracle.cells_tree(g_hi[k].numpy(), g_comp[k].numpy()) for k in range(3)]
        want = [oracle.cells_finish(hi_all[k], comp_all[k]) for k in range(3)]
        queue.put((rank, got, want, base, count))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [131072 * 3 + 5000, 4096 * 32 * 2, 1000])
def test_two_ranks_gather_leaves_bit_identical_to_one(n):
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shards = sorted((r[3], r[4]) for r in results)
    assert shards[0][0] == 0 and shards[0][0] + shards[0][1] == shards[1][0]
    assert shards[1][0] + shards[1][1] == n
    assert shards[0][1] % sharded.LEAF_SAMPLES == 0 or shards[1][1] == 0
    for rank, got, want, _b, _c in results:
        assert got == want, (rank, got, want)


def test_shard_ranges_cover_and_align():
    for n in (1, 131071, 131072, 131073, 10 ** 7):
        for world in (1, 2, 3, 4, 8):
            cuts = [sharded.shard_range(n, world, r) for r in range(world)]
            pos = 0
            for base, count in cuts:
                assert base == pos and count >= 0
                pos += count
                if base + count < n:
                    assert (base + count) % sharded.LEAF_SAMPLES == 0
            assert pos == n


@pytest.mark.parametrize("world,per", [(2, 4), (4, 8), (8, 1), (3, 16), (8, 512)])
@pytest.mark.parametrize("op", ["sum", "max", "min"])
def test_aligned_subtrees_finish_like_one_tree(world, per, op):
    """When every rank holds the same power-of-two number of leaves, its leaves
    are an aligned subtree of the one-device tree: the ranks' subtree roots
    (hi, comp), joined by the same pairwise levels, give the one tree's cell
    bit for bit (the exchange ``sharded.finish_subtrees`` runs on the device)."""
    import oracle

    rng = np.random.default_rng(world * 1000 + per)
    n = world * per
    hi = rng.standard_normal(n) * np.exp(rng.uniform(-30, 30, n))
    comp = hi * rng.standard_normal(n) * 1e-17 if op == "sum" else np.zeros(n)
    assert sharded.aligned([per] * world)
    roots = [oracle.cells_tree_pair(hi[r * per:(r + 1) * per], comp[r * per:(r + 1) * per], op) for r in range(world)]
    rh = np.array([h for h, _c in roots])
    rc = np.array([c for _h, c in roots])
    assert oracle.cells_tree(rh, rc, op) == oracle.cells_tree(hi, comp, op)


def test_unequal_or_odd_leaf_counts_take_the_full_gather():
    assert not sharded.aligned([4, 4, 3])
    assert not sharded.aligned([6, 6])
    assert not sharded.aligned([0, 0])
    assert sharded.aligned([16, 16, 16])


def test_shard_counts_follow_the_cut():
    for n in (1, 131072, 131073, 3 * 131072 + 5, 10 ** 7):
        for world in (1, 2, 3, 8):
            counts = sharded.shard_counts(n, world)
            assert counts == [sharded.leaves_of(sharded.shard_range(n, world, r)[1])
                              if sharded.shard_range(n, world, r)[1] else 0 for r in range(world)]
            assert sum(counts) == sharded.leaves_of(n)


def _leaving_rank_main(rank, world, port, queue):
    """Rank 1 takes part in the first step's gather and then leaves (between
    steps, nothing of its own in flight); rank 0 goes on to the second step's
    gather, which must end with an error inside the group's timeout."""
    import datetime
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    lh = torch.full((3, 2), float(rank))
    lc = torch.zeros((3, 2))
    sharded.gather_leaves(lh, lc, [2] * world)
    if rank == 1:
        queue.put((rank, "left", 0.0))
        queue.close()
        queue.join_thread()
        os._exit(0)                      # leaves without another collective
    t0 = time.monotonic()
    try:
        sharded.gather_leaves(lh, lc, [2] * world)
        queue.put((rank, "no error", time.monotonic() - t0))
    except Exception as exc:            # noqa: BLE001 -- the error is the result
        queue.put((rank, f"error: {type(exc).__name__}", time.monotonic() - t0))
    queue.close()
    queue.join_thread()
    os._exit(0)


def test_a_rank_that_leaves_between_steps_ends_the_others_next_gather_with_an_error():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results[1][1] == "left"
    assert results[0][1].startswith("error"), results
    assert results[0][2] < 60.0, results


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_leaf_stage_and_tree_are_the_finish(dtype):
    """The oracle's finish split where the ranks split it: leaf partials, then
    the tree over them, equal the one-pass finish bit for bit (both types)."""
    import oracle

    rng = np.random.default_rng(5)
    n = 3 * 131072 + 777
    x = rng.uniform(-2, 2, n).astype(dtype)
    t = (x + 0.1 * rng.standard_normal(n)).astype(dtype)
    hi, comp = oracle.poly_loss_vjp_rows(x, t, np.ones(n, dtype=dtype), dtype(0.5), dtype(-1.0), dtype(2.0))
    for k in range(3):
        lh, lc = oracle.cells_leaves(hi[k], comp[k])
        assert lh.dtype == dtype and lh.shape[0] == sharded.leaves_of(n)
        assert oracle.cells_tree(lh, lc) == oracle.cells_finish(hi[k], comp[k])
