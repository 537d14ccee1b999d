"""Multi-GPU plumbing of the sharded BrFS (no counterpart in maichmueller/mymyr, which has no multi-GPU layer).

One process per GPU, launched by torchrun. ``Communicator(ctx)`` builds the ranks' NCCL communicator of the device
library from a ``torch.distributed`` process group (rank 0 makes the NCCL id, the group broadcasts it);
``cuda.brfs(task, comm=comm)`` then runs the search sharded by state-hash owner, with every rank calling it together.
``gather_states`` assembles the ranks' states in id order (for checks and exports; the search itself never gathers).

    torch.distributed.init_process_group("nccl")
    ctx = mymyr_b200.Context(local_rank)
    comm = dist.Communicator(ctx)
    r = cuda.brfs(Task.from_text(text, ctx), comm=comm, stop_at_goal=False)
    states = dist.gather_states(r)            # every rank: ids, rows, hashes, parent, index in id order
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import check, lib
from .task import Context


def new_comm_id() -> bytes:
    """A fresh NCCL id (128 bytes) for a communicator; made on one rank and handed to all."""
    cid = _lib.CommId()
    check(lib().b2_comm_id_new(C.byref(cid)))
    return C.string_at(C.addressof(cid), C.sizeof(cid))


def broadcast_comm_id(group=None) -> bytes:
    """Rank 0 of the torch.distributed group makes an NCCL id; every rank returns it."""
    import torch.distributed as tdist

    src = tdist.get_global_rank(group, 0) if group is not None else 0
    obj = [new_comm_id() if tdist.get_rank(group) == 0 else None]
    tdist.broadcast_object_list(obj, src=src, group=group)
    return obj[0]


class Communicator:
    """The device library's communicator over the ranks of a torch.distributed group (collective to create).
    ``timeout_s``: how long a rank waits for the others in a collective before it fails the search (default 600)."""

    def __init__(self, ctx: Context, group=None, comm_id: bytes | None = None, timeout_s: float | None = None):
        import torch.distributed as tdist

        self.ctx = ctx
        self.rank = tdist.get_rank(group)
        self.world = tdist.get_world_size(group)
        cid_bytes = comm_id if comm_id is not None else broadcast_comm_id(group)
        if len(cid_bytes) != C.sizeof(_lib.CommId):
            raise ValueError("Communicator: an NCCL id has 128 bytes")
        cid = _lib.CommId()
        C.memmove(C.addressof(cid), cid_bytes, len(cid_bytes))
        h = C.c_void_p()
        check(lib().b2_comm_create(ctx.handle, C.byref(cid), self.rank, self.world, C.byref(h)))
        self._h = h
        if timeout_s is not None:
            check(lib().b2_comm_set_timeout(h, float(timeout_s)))

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.b2_comm_destroy(h)
        self._h = None

    def __del__(self):
        self.close()


def merge_shards(shards: list[dict]) -> dict:
    """The union of the ranks' local state lists (each in id order, ids disjoint), in id order. Raises if the ids are
    not exactly 0..n-1 (a state lost or stored twice)."""
    keys = [k for k in ("ids", "rows", "hashes", "parent", "index") if all(k in s for s in shards)]
    cat = {k: np.concatenate([np.asarray(s[k]) for s in shards]) for k in keys}
    order = np.argsort(cat["ids"], kind="stable")
    out = {k: v[order] for k, v in cat.items()}
    ids = out["ids"]
    if not np.array_equal(ids, np.arange(len(ids), dtype=ids.dtype)):
        raise RuntimeError("gather_states: the ranks' ids are not a partition of 0..n-1")
    return out


def gather_states(result, group=None, *, rows: bool = True, hashes: bool = True, nodes: bool = True) -> dict:
    """Every rank's states (``BrfsResult.local``) gathered on every rank of the group, in id order."""
    import torch.distributed as tdist

    local = result.local(rows=rows, hashes=hashes, nodes=nodes)
    shards: list = [None] * tdist.get_world_size(group)
    tdist.all_gather_object(shards, local, group=group)
    return merge_shards(shards)
