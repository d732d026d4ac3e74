"""Samples sharded across GPUs: one process per GPU, one exchange for cells.

Every kernel here is sample-local (each sample reads and writes only its own
column), so samples shard with no communication: rank ``r`` of ``world`` runs
the contiguous range ``shard_range(n, world, r)`` -- the reference's rank cut
is contiguous too (tests/mpi/test_hawk_rank_oracle.py:94-168).  The one
exchange is for cells (sample sums such as Param gradients):

1. each rank writes the 32-sample rows of its shard and folds them into one
   (hi, comp) partial per leaf of 4096 rows (``hkb_cells_leaves``);
2. when every rank holds the same power-of-two number of leaves, each folds
   its own leaves to one (hi, comp) pair per column (an aligned subtree of the
   one-device tree), the ranks all-gather the pairs and every rank runs the
   last levels over them -- with a ``PeerFinish``, all of it in one launch that
   stores each rank's pairs into every rank's memory over NVLink; otherwise
   the ranks all-gather their leaf partials (NCCL over NVLink on B200s)
3. and every rank folds all leaves in rank order with the same pairwise tree
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


def aligned(counts) -> bool:
    """Whether every rank holds the same power-of-two number of leaves: then each
    rank's leaves are an aligned subtree of the one-device tree."""
    first = counts[0]
    return first > 0 and (first & (first - 1)) == 0 and all(c == first for c in counts)


class PeerFinish:
    """The last step of ``finish_subtrees`` over NVLink peer memory in one
    launch per call (``hkb_peer_finish``), in place of the NCCL all-gather
    between two tree launches: each rank folds its leaves to one root per
    column, stores the root into every rank's exchange area (plain peer stores
    through CUDA IPC mappings, each 32-bit half in a word beside the round's
    tag), waits (bounded, two seconds) until every rank's words of the round
    carry the tag, and folds the roots in rank order -- the same tree, bit for
    bit.

    Made collectively (every rank of ``group``, once): each rank allocates its
    area on ``device`` and the ranks exchange the areas' IPC handles
    (``all_gather_object``).  Every call after that is collective too, in the
    same order on every rank (rounds are numbered by the call).  A wait that
    ran out leaves the cells unwritten and is reported by ``check``;
    ``close`` (collective: a barrier first, so no rank still stores into an
    area) frees the area."""

    def __init__(self, mode: str, cols: int, device: int, group=None) -> None:
        import torch.distributed as dist

        from . import abi

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.mode, self.cols = mode, cols
        self.area = abi.PeerArea(device, self.rank, self.world, mode, cols)
        handles = [None] * self.world
        dist.all_gather_object(handles, self.area.handle, group=group)
        self.area.connect(handles)
        self.seq = 0

    def finish(self, op: str, leaf_hi, leaf_comp, leaves: int, values, stream: int = 0,
               timeout_ns: int = 0) -> None:
        """The cells of every column over every rank's ``leaves`` partials of
        ``leaf_hi`` / ``leaf_comp`` (``(cols, leaves)``, folded in place) into
        ``values``, on ``stream``."""
        from .errors import HawkError

        if leaf_hi.shape[0] < self.cols or values.numel() < self.cols:
            raise HawkError(f"the peer finish was made for {self.cols} columns")
        self.seq += 1
        if self.seq & 0xFFFFFFFF == 0:      # a round's tag is its low 32 bits; tag 0 is a fresh area's
            self.seq += 1
        self.area.finish(op, leaf_hi.data_ptr(), leaf_comp.data_ptr(), leaves, values.data_ptr(), self.seq,
                         timeout_ns, stream)

    def check(self) -> None:
        """Read (synchronising) and clear the area's status word; a wait that
        ran out raises ``HawkError``."""
        from . import abi
        from .errors import HawkError

        flags = self.area.status()
        if flags & abi.PEER_TIMEOUT:
            raise HawkError(f"rank {self.rank}: a peer finish waited past its limit for another rank's root "
                            "(the cells of that call were not written)")

    def close(self) -> None:
        import torch.distributed as dist

        dist.barrier(self.group)
        self.area.free()


def finish_subtrees(op: str, mode: str, cols: int, leaf_hi, leaf_comp, leaves: int, values, group=None,
                    stream: int = 0, pack=None, gathered=None, peer: PeerFinish | None = None) -> None:
    """The cells of ``cols`` columns from every rank's ``leaves`` partials
    (``(cols, leaves)`` tensors; ``leaves`` a power of two, the same on every
    rank), into ``values``: this rank's tree over its own leaves to one (hi,
    comp) pair per column, an all-gather of the pairs (``world * cols * 2``
    values over NVLink), and the last pairwise levels over the ranks' roots.
    The pairwise levels of the one-device tree over ``world * leaves`` leaves
    join each rank's leaves among themselves first, so this is the same tree,
    bit for bit (hawk/_cells.py:108-119).  ``pack`` ``(2, cols)`` and
    ``gathered`` ``(world, 2, cols)`` may be passed preallocated.  With
    ``peer`` the three steps are one ``PeerFinish`` launch over peer memory."""
    import torch
    import torch.distributed as dist

    from . import abi

    if peer is not None:
        peer.finish(op, leaf_hi, leaf_comp, leaves, values, stream)
        return
    world = dist.get_world_size(group)
    if pack is None:
        pack = torch.empty((2, cols), dtype=leaf_hi.dtype, device=leaf_hi.device)
    if gathered is None:
        gathered = torch.empty((world, 2, cols), dtype=leaf_hi.dtype, device=leaf_hi.device)
    item = leaf_hi.element_size()
    abi.cells_tree_ex(op, mode, cols, leaf_hi.data_ptr(), leaf_comp.data_ptr(), leaves, 1, leaves,
                      pack.data_ptr(), pack.data_ptr() + cols * item, stream)
    dist.all_gather_into_tensor(gathered, pack, group=group)
    abi.cells_tree_ex(op, mode, cols, gathered.data_ptr(), gathered.data_ptr() + cols * item, world, 2 * cols, 1,
                      values.data_ptr(), 0, stream)


def shard_counts(total_samples: int, world: int) -> list:
    """Every rank's leaf count when ``total_samples`` are cut by ``shard_range``."""
    return [leaves_of(shard_range(total_samples, world, r)[1]) if shard_range(total_samples, world, r)[1] else 0
            for r in range(world)]


def run_cells(kernel, *, group=None, base: int = 0, count: int | None = None, n_samples: int | None = None,
              total_samples: int | None = None, stream=None, peer: PeerFinish | None = None, **arrays) -> None:
    """``hawk_b200.runtime.run`` of a kernel with cells over this rank's shard,
    its cells summed over the samples of every rank of ``group``.

    Each rank binds its own shard's planes (``n_samples`` local samples, a
    multiple of 131072 on every rank but the last); the cells every rank
    receives are bit-identical to one GPU's over the concatenated shards.

    ``total_samples``: the sample count of the whole job, cut over the ranks by
    ``shard_range``.  Every rank's leaf count then follows from it, so the call
    makes one collective (the partials) and no host round trip; this rank's
    shard must be the one ``shard_range`` gives it (refused otherwise).  Without
    it the ranks first exchange their leaf counts (a second collective, read
    back on the host).

    Every launch and every collective is ordered on ``stream`` (the current
    stream when None): the partials are gathered after the kernels that write
    them, and the final tree runs after the gather lands.  ``peer``: a
    ``PeerFinish`` of this group for the kernel's columns, used where every
    rank holds the same power-of-two leaf count (else the gather runs)."""
    import torch
    import torch.distributed as dist

    from . import runtime
    from .errors import HawkError

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
            with torch.cuda.stream(runtime._torch_stream(stream, kernel.device)):
                if total_samples is not None:
                    rank = dist.get_rank(group)
                    want = shard_range(int(total_samples), world, rank)[1]
                    if hi - lo != -(-want // ROW):
                        raise HawkError(f"rank {rank}: its shard holds {hi - lo} rows of 32 samples but "
                                        f"shard_range({total_samples}, {world}, {rank}) gives it {want} samples")
                    counts = shard_counts(int(total_samples), world)
                else:
                    counts_t = torch.tensor([leaves], dtype=torch.int64, device=f"cuda:{kernel.device}")
                    every = torch.zeros(world, dtype=torch.int64, device=f"cuda:{kernel.device}")
                    dist.all_gather_into_tensor(every, counts_t, group=group)
                    counts = [int(c) for c in every.cpu().tolist()]
                if aligned(counts):
                    op = kernel.sums[0]["op"] if kernel.sums else "sum"
                    finish_subtrees(op, kernel.element, cols, state["leaf_hi"], state["leaf_comp"], leaves,
                                    state["values"], group, runtime._stream(stream, kernel.device), peer=peer)
                    kernel.write_cells(state["values"], outputs, stream)
                    return
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
