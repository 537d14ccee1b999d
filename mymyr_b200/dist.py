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


class RankLeft(RuntimeError):
    """A rank of the communicator has left it: a search over it is not started."""


class Membership:
    """Which ranks are still in a communicator, kept in a torch.distributed Store under `key`: a rank that leaves
    says so (leave()), and every rank checks before a search's first launch (check(): one store round trip), so that
    the others fail on the host, with no kernel or collective in flight, instead of waiting in a collective for a
    rank that is gone. A rank that dies without leaving is caught by the communicator's timeout instead."""

    def __init__(self, store, key: str, rank: int):
        self.store, self.key, self.rank = store, key, rank
        self.left = False

    def leave(self) -> None:
        if not self.left:
            self.left = True
            self.store.set(f"{self.key}/left/{self.rank}", b"1")
            self.store.add(f"{self.key}/left", 1)

    def check(self) -> None:
        n = int(self.store.add(f"{self.key}/left", 0))
        if n:
            raise RankLeft(f"mymyr_b200: {n} rank(s) left the communicator ({self.key}); the search is not started")


def default_store():
    """The default process group's store (None when torch.distributed keeps none)."""
    try:
        from torch.distributed import distributed_c10d

        return distributed_c10d._get_default_store()
    except Exception:
        return None


class Communicator:
    """The device library's communicator over the ranks of a torch.distributed group (collective to create).
    ``timeout_s``: how long a rank waits for the others in a collective before it fails the search (default 600).
    ``store``: where the ranks record that they left (default: the default process group's store); a search over a
    communicator that a rank has left raises RankLeft on the other ranks before it launches anything."""

    def __init__(self, ctx: Context, group=None, comm_id: bytes | None = None, timeout_s: float | None = None,
                 store=None):
        import torch.distributed as tdist

        self.ctx = ctx
        self.rank = tdist.get_rank(group)
        self.world = tdist.get_world_size(group)
        cid_bytes = comm_id if comm_id is not None else broadcast_comm_id(group)
        if len(cid_bytes) != C.sizeof(_lib.CommId):
            raise ValueError("Communicator: an NCCL id has 128 bytes")
        cid = _lib.CommId()
        C.memmove(C.addressof(cid), cid_bytes, len(cid_bytes))
        store = store if store is not None else default_store()
        self.members = Membership(store, "b2comm/" + cid_bytes[:16].hex(), self.rank) if store is not None else None
        h = C.c_void_p()
        check(lib().b2_comm_create(ctx.handle, C.byref(cid), self.rank, self.world, C.byref(h)))
        self._h = h
        if timeout_s is not None:
            check(lib().b2_comm_set_timeout(h, float(timeout_s)))

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def check(self) -> None:
        """Raises RankLeft if a rank has left the communicator (every search over it calls this first)."""
        if self._h is None:
            raise RankLeft("mymyr_b200: this rank's communicator is closed")
        if self.members is not None:
            self.members.check()

    def leave(self) -> None:
        """Announces between searches that this rank takes part in no further search: the other ranks' next search
        over the communicator raises RankLeft before it launches anything. Not collective; close() still is."""
        members = getattr(self, "members", None)
        if members is not None:
            try:
                members.leave()
            except Exception:  # the store may be gone at interpreter exit
                pass

    def close(self) -> None:
        """Leaves the communicator and releases it. Collective: every rank closes it (NCCL's communicator teardown
        waits for the other ranks), after any search over it has ended on every rank."""
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            self.leave()
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
