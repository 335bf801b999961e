"""How the sharded paths split their work across ranks (one process per
GPU) and which collective finishes each result.

- Reductions split over the leading axis (config 2): rank r owns rows
  [r*n/P, (r+1)*n/P) of axis 0.  A reduction that keeps axis 0 is final on
  each rank and its pieces are concatenated in rank order (all-gather); one
  that folds axis 0 leaves a partial per rank, finished by an all-reduce with
  the same fold (exact for min/max; a sum reorders the terms).
- Data-parallel training (config 4): the global batch is split into equal
  contiguous pieces; the loss is scaled by the global batch, so the sum of
  the ranks' gradients is the gradient of the whole batch.
"""
from __future__ import annotations


def shard(extent: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank `rank`'s share of `extent` rows: contiguous,
    the first `extent % world` ranks one row longer."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, extra = divmod(extent, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def finishing_collective(axes, sharded_axis: int = 0) -> str:
    """'allgather' when the reduction keeps the sharded axis (results are
    concatenated), 'allreduce' when it folds it (partials are combined)."""
    return "allreduce" if sharded_axis in axes else "allgather"


def batch_split(global_batch: int, world: int) -> int:
    if global_batch % world:
        raise ValueError(f"a global batch of {global_batch} does not split over {world} ranks")
    return global_batch // world


def nccl_comm(torch, world: int, rank: int):
    """The library's NCCL communicator for this rank (None at world 1):
    rank 0 draws the unique id and torch.distributed broadcasts it."""
    import ctypes as C

    from . import _native as N
    if world == 1:
        return None
    uid = (C.c_uint8 * 128)()
    if rank == 0:
        N.call("tc_comm_unique_id", uid)
    t = torch.tensor(list(uid), dtype=torch.uint8, device="cuda")
    torch.distributed.broadcast(t, 0)
    uid = (C.c_uint8 * 128)(*t.cpu().tolist())
    comm = C.c_void_p()
    N.call("tc_comm_init", rank, world, uid, C.byref(comm))
    return comm


class PeerBuffer:
    """A tc_peer_buffer: `nbytes` on every rank, each mapping the others'."""

    def __init__(self, comm, nbytes: int):
        import ctypes as C

        from . import _native as N
        self.handle = C.c_void_p()
        N.call("tc_peer_buffer_create", comm, nbytes, C.byref(self.handle))
        local = C.c_void_p()
        N.call("tc_peer_buffer_pointer", self.handle, C.byref(local))
        self.ptr, self.nbytes = local.value, nbytes

    def close(self) -> None:
        from . import _native as N
        if self.handle:
            N.call("tc_peer_buffer_destroy", self.handle)
            self.handle = None
