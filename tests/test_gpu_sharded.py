"""Cells over samples sharded across GPUs, one process per GPU over NCCL.

Each rank binds its contiguous shard (``sharded.shard_range``), writes its
32-sample rows, folds them into leaf partials, all-gathers the partials and
runs the same pairwise tree; every rank's Param gradients must be
bit-identical to the oracle's finish over all samples (hawk/_cells.py:94-119
over the unsharded rows).  Two call forms: the leaf counts exchanged by the
ranks on the current stream, and the counts derived from the job's sample
count (``total_samples``) with every launch and collective on a side stream;
and, with every rank on aligned subtrees, the last step over NVLink peer
memory (``sharded.PeerFinish``, several rounds so both round parities of the
exchange area are used).  A rank that leaves a round of the peer finish makes
the other's bounded wait run out: that rank's cells stay unwritten, the status
reports it, and the next round both join is bit-identical again.  NVLS is off
(``NCCL_NVLS_ENABLE=0``).  Skipped with fewer GPUs than ranks.
"""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest

import oracle
from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

BUNDLES = REPO / "hawk_b200" / "bundles"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, form, queue):
    import torch.distributed as dist

    from hawk_b200 import runtime, sharded, workloads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = workloads.poly_loss(n, seed=n)
        base, count = sharded.shard_range(n, world, rank)

        def dev(a):
            return torch.as_tensor(np.ascontiguousarray(a), device=f"cuda:{rank}")

        sl = slice(base, base + count)
        cells = {k: torch.full((1,), float("nan"), dtype=torch.float64, device=f"cuda:{rank}")
                 for k in ("bar_a", "bar_b", "bar_c")}
        abc = {k: dev(np.array([w[k]])) for k in ("a", "b", "c")}
        vjp = runtime.load(BUNDLES, "poly_loss_vjp", "float64", rank)
        planes = dict(x=dev(w["x"][sl]), t=dev(w["t"][sl]), bar_r=dev(w["bar_r"][sl]), **abc, **cells)
        if form == "side stream":
            side = torch.cuda.Stream(device=rank)
            side.wait_stream(torch.cuda.current_stream(rank))
            for _ in range(2):          # the second call's finish reuses the first's scratch
                sharded.run_cells(vjp, total_samples=n, stream=side, **planes)
            side.synchronize()
        elif form == "peer memory":
            peer = sharded.PeerFinish("float64", 3, rank)
            for _ in range(3):          # rounds 1, 2, 3: both parities of the exchange area
                for k in ("bar_a", "bar_b", "bar_c"):
                    cells[k].fill_(float("nan"))
                sharded.run_cells(vjp, total_samples=n, peer=peer, **planes)
            torch.cuda.synchronize(rank)
            peer.check()
            peer.close()
        else:
            sharded.run_cells(vjp, **planes)
        torch.cuda.synchronize(rank)
        queue.put((rank, base, count, [float(cells[k].cpu()[0]) for k in ("bar_a", "bar_b", "bar_c")]))
    finally:
        dist.destroy_process_group()


def _worlds():
    count = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [w for w in (2, 4, 8) if w <= max(count, 2)]


@pytest.mark.parametrize("form", ["counts exchanged", "side stream", "peer memory"])
@pytest.mark.parametrize("shape", ["ragged", "aligned"])
@pytest.mark.parametrize("world", _worlds())
def test_sharded_param_gradients_bit_identical_to_one_device(world, shape, form):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    if form == "peer memory" and shape == "ragged":
        pytest.skip("the peer finish joins aligned subtrees; ragged shards gather their leaves")
    import torch.multiprocessing as mp

    from hawk_b200 import sharded, workloads

    # ragged: every rank holds at least one leaf and the last shard is short (the
    # full gather of leaf partials); aligned: 4 leaves on every rank (each rank's
    # subtree root is exchanged, sharded.finish_subtrees)
    n = 2 * world * sharded.LEAF_SAMPLES - 1000 if shape == "ragged" else 4 * world * sharded.LEAF_SAMPLES
    w = workloads.poly_loss(n, seed=n)
    want, _rows = oracle.poly_loss_vjp(w["x"], w["t"], w["bar_r"], w["a"], w["b"], w["c"])
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, form, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results.sort()
    assert sum(r[2] for r in results) == n
    for rank, _base, count, got in results:
        assert count > 0
        assert got == [float(v) for v in want], (rank, got, want)


def _skip_main(rank, world, port, queue):
    """Two ranks on the exchange area directly: the second exchange is rank 0's alone."""
    import torch.distributed as dist

    from hawk_b200 import abi

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        area = abi.PeerArea(rank, rank, world, "float64", 1)
        handles = [None] * world
        dist.all_gather_object(handles, area.handle)
        area.connect(handles)
        out = {}
        for seq in (1, 2, 3):
            if seq == 2 and rank == 1:
                continue                                    # rank 1 leaves the second exchange
            hi = torch.tensor([[1.0 + rank + seq]], dtype=torch.float64, device=f"cuda:{rank}")
            comp = torch.zeros_like(hi)
            cell = torch.full((1,), float("nan"), dtype=torch.float64, device=f"cuda:{rank}")
            area.finish("sum", hi.data_ptr(), comp.data_ptr(), 1, cell.data_ptr(), seq,
                        timeout_ns=100_000_000 if seq == 2 else 0)
            torch.cuda.synchronize(rank)
            out[seq] = (float(cell.cpu()[0]), area.status())
        dist.barrier()
        area.free()
        queue.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_a_rank_that_leaves_a_round_is_reported_and_the_next_round_joins():
    if torch.cuda.device_count() < 2:
        pytest.skip(f"needs 2 GPUs, {torch.cuda.device_count()} visible")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_skip_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # round r: rank k's root is 1 + k + r, the cell their sum
    for rank in (0, 1):
        assert results[rank][1] == (5.0, 0) and results[rank][3] == (9.0, 0)
    cell, status = results[0][2]
    assert np.isnan(cell) and status == 1          # rank 0 waited past its limit, its cell unwritten
    assert 2 not in results[1]
