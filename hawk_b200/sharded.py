"""Samples sharded across GPUs: one process per GPU, one exchange for cells.

Every kernel here is sample-local (each sample reads and writes only its own
column), so samples shard with no communication: rank ``r`` of ``world`` runs
the contiguous range ``shard_range(n, world, r)`` -- the reference's rank cut
is contiguous too (tests/mpi/test_hawk_rank_oracle.py:94-168).  The one
exchange is for cells (sample sums such as Param gradients):

1. each rank writes the 32-sample rows of its shard and folds them into one
   (hi, comp) partial per leaf of 4096 rows (``hkb_cells_leaves``);
2. the ranks all-gather their leaf partials (NCCL over NVLink on B200s);
3. every rank folds all leaves in rank order with the same pairwise tree
   (``hkb_cells_tree``).

Shards start on leaf boundaries (4096 rows = 131072 samples), so the gathered
leaves are exactly the leaves of the unsharded row array and every rank's
cells are bit-identical to a single GPU's over all samples
(hawk/_cells.py:94-119 is the tree).  All ranks take the same collective steps
in the same order.
"""

from __future__ import annotations

ROW = 32
LEAF_ROWS = 4096
LEAF_SAMPLES = ROW * LEAF_ROWS


def shard_range(n: int, world: int, rank: int) -> tuple:
    """``(base, count)`` of rank ``rank``: contiguous, starting on a leaf
    boundary; the last rank takes the remainder (possibly empty shards at the
    end when ``n`` is small)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    leaves = -(-n // LEAF_SAMPLES)
    per = -(-leaves // world)
    base = min(rank * per * LEAF_SAMPLES, n)
    end = min((rank + 1) * per * LEAF_SAMPLES, n)
    return base, end - base


def leaves_of(samples: int) -> int:
    rows = -(-samples // ROW)
    return -(-rows // LEAF_ROWS)


def gather_leaves(leaf_hi, leaf_comp, counts, group=None):
    """All-gather every rank's leaf partials and lay them out column-major.

    ``leaf_hi``/``leaf_comp`` are this rank's ``(cols, L_r)`` tensors padded to
    ``(cols, max(counts))``; ``counts[r]`` is rank r's leaf count.  Returns
    ``(hi, comp)`` of shape ``(cols, sum(counts))``: column k's leaves of rank
    0, then rank 1, ... -- the leaf order of the unsharded rows."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    cols, width = leaf_hi.shape
    packed = torch.stack([leaf_hi, leaf_comp]).contiguous()          # (2, cols, width)
    out = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(out, packed, group=group)
    parts = [out[r][:, :, :counts[r]] for r in range(world) if counts[r] > 0]
    both = torch.cat(parts, dim=2).contiguous()                      # (2, cols, total)
    return both[0].contiguous(), both[1].contiguous()


def run_cells(kernel, *, group=None, base: int = 0, count: int | None = None, n_samples: int | None = None,
              stream=None, **arrays) -> None:
    """``hawk_b200.runtime.run`` of a kernel with cells over this rank's shard,
    its cells summed over the samples of every rank of ``group``.

    Each rank binds its own shard's planes (``n_samples`` local samples, a
    multiple of 131072 on every rank but the last); the cells every rank
    receives are bit-identical to one GPU's over the concatenated shards."""
    import torch
    import torch.distributed as dist

    from . import runtime

    with kernel._lock:
        pending = runtime.launch_cells(kernel, base=base, count=count, n_samples=n_samples, stream=stream,
                                       **arrays)
        if pending is None:
            return
        state, outputs, lo, hi = pending
        cols = len(kernel.sums)
        leaves = kernel.cells_leaves(state, lo, hi, stream) if hi > lo else 0
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        if world > 1:
            counts_t = torch.tensor([leaves], dtype=torch.int64, device=f"cuda:{kernel.device}")
            every = [torch.zeros_like(counts_t) for _ in range(world)]
            dist.all_gather(every, counts_t, group=group)
            counts = [int(c.item()) for c in every]
            width = max(max(counts), 1)
            flat_hi = state["leaf_hi"].view(-1)
            flat_comp = state["leaf_comp"].view(-1)
            pad = torch.zeros((2, cols, width), dtype=flat_hi.dtype, device=flat_hi.device)
            if leaves:
                pad[0, :, :leaves] = flat_hi[:cols * leaves].view(cols, leaves)
                pad[1, :, :leaves] = flat_comp[:cols * leaves].view(cols, leaves)
            all_hi, all_comp = gather_leaves(pad[0], pad[1], counts, group)
            total = all_hi.shape[1]
        else:
            all_hi, all_comp, total = state["leaf_hi"], state["leaf_comp"], leaves
        if total:
            kernel.cells_tree(all_hi, all_comp, total, state["values"], stream)
            kernel.write_cells(state["values"], outputs, stream)
