"""The multi-GPU path on the CPU: gloo ranks (world size 2 and 3) run the sharded BrFS protocol of dbrfs.cu step for
step, with the reference's own successor generator, and must reproduce the reference's deterministic ids, node
records and layer counts; the NCCL id broadcast and the gathering of the ranks' shards run over gloo as well.

The protocol model here is test infrastructure: it mirrors the device kernels' decisions (owner by hash; per-parent
successor counts in byte lanes, widened to word lanes once a count overflows, all-reduced and scanned into candidate
offsets; records keyed parent id << 32 | successor index; the smallest key per state at its owner; ids by popcount
prefixes of the all-reduced candidate bitmap; node records from the key) so that a flaw in the partition logic shows
without a GPU.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as td
import torch.multiprocessing as mp

from mymyr_b200 import dist as bdist
from mymyr_b200 import tasks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world)


def owner_of(h: int, world: int) -> int:
    """dev::owner_of: the hash's high 32 bits scaled to [0, world)."""
    return ((int(h) >> 32) * world) >> 32


def sharded_brfs_model(text: str, rank: int, world: int, max_depth: int | None, witness: bool = True,
                       shard_from: int = 1) -> dict:
    """One rank of the sharded BrFS protocol (dbrfs.cu); successors from the compiled reference (rl::expand). With
    shard_from > 1 every rank first runs the same one-GPU search alone (here the reference's BrFS) up to the first
    layer of at least shard_from new states, keeps the states it owns (id order, global parent ids) and goes on from
    there, as shard_run does after run_prefix."""
    from oracle import ref as oref

    t = oref.RefTask(text)
    root = t.initial_state()
    h0 = oref.hash_state(root)
    store: dict[bytes, int] = {}          # this rank's states: row bytes -> id
    mine: list[tuple[int, np.ndarray, int, int]] = []  # (id, row, parent, index), id order
    if owner_of(h0, world) == rank:
        store[root.tobytes()] = 0
        mine.append((0, root, 0xFFFFFFFF, 0))
    layer_begin, layer_end, n_total, lb_local = 0, 1, 1, 0
    counts = []
    layers = 0
    lane = 1
    if shard_from > 1:
        full = t.brfs(max_depth=max_depth, stop_at_goal=False, witness_pruning=witness)["layer_counts"]
        cut = next((L for L, (_, _, n) in enumerate(full) if n >= shard_from and (max_depth is None or L + 1 < max_depth)),
                   None)
        if cut is not None:
            rows, par, idx = t.brfs_states(max_depth=cut + 1, witness_pruning=witness)
            counts = [tuple(c) for c in full[: cut + 1]]
            layers = cut + 1
            n_total = len(rows)
            layer_end = n_total
            layer_begin = n_total - counts[-1][2]
            store.clear()
            mine.clear()
            for sid in range(n_total):  # the conversion: owned states in id order
                if owner_of(oref.hash_state(rows[sid]), world) == rank:
                    store[rows[sid].tobytes()] = sid
                    mine.append((sid, rows[sid].copy(), 0xFFFFFFFF if sid == 0 else int(par[sid]), int(idx[sid])))
            lb_local = next((i for i, m in enumerate(mine) if m[0] >= layer_begin), len(mine))
    while layer_end > layer_begin and (max_depth is None or layers < max_depth):
        layers += 1
        E = layer_end - layer_begin
        frontier = mine[lb_local:]
        rows = np.array([r for _, r, _, _ in frontier], np.uint64).reshape(-1, t.words)
        ex = t.expand(rows, witness_pruning=witness, succ=True) if len(frontier) else None
        # k_dscatter: byte lanes by parent id (saturated at 255 and counted), or word lanes once a layer overflowed
        local_counts = [int(ex["offsets"][i + 1] - ex["offsets"][i]) for i in range(len(frontier))]
        while True:
            cg = torch.zeros(E + 1, dtype=torch.int64)  # lanes, then the overflow count
            for i, (pid, _, _, _) in enumerate(frontier):
                c = local_counts[i]
                if lane == 1 and c > 255:
                    cg[E] += 1
                    c = 255
                cg[pid - layer_begin] = c
            td.all_reduce(cg)
            if lane == 1 and int(cg[E]):
                lane = 4  # every rank sees the same sum, so all of them redo the layer with word lanes
                continue
            break
        gbase = np.concatenate([[0], np.cumsum(cg.numpy()[:E])]).astype(np.int64)
        G = int(gbase[-1])
        # stage [row | hash | key] per local successor, key = parent id << 32 | successor index; the exchange (a
        # peer-memory push on the device) is an all-gather here, each owner keeping its bucket
        records = []
        for i, (pid, _, _, _) in enumerate(frontier):
            for k in range(int(ex["offsets"][i]), int(ex["offsets"][i + 1])):
                h = int(ex["succ_hash"][k])
                records.append((owner_of(h, world), ex["succ"][k].tobytes(), (pid << 32) | (k - int(ex["offsets"][i]))))
        everyone: list = [None] * world
        td.all_gather_object(everyone, records)
        best: dict[bytes, int] = {}  # k_dinsert: the smallest key of each new state of this owner
        for recs in everyone:
            for d, row, key in recs:
                if d != rank or row in store:
                    continue
                if row not in best or key < best[row]:
                    best[row] = key
        # k_dmark: bit c = gbase[parent] + successor index of each new state, in 32-bit words
        nw = (G + 31) // 32
        fm = torch.zeros(max(nw, 1), dtype=torch.int64)
        cand = {}
        for row, key in best.items():
            c = int(gbase[(key >> 32) - layer_begin] + (key & 0xFFFFFFFF))
            assert not (int(fm[c >> 5]) >> (c & 31)) & 1, "two states share a candidate index"
            fm[c >> 5] += 1 << (c & 31)
            cand[row] = c
        f = fm.clone()
        td.all_reduce(f)
        assert all(int(x) < (1 << 32) for x in f), "two owners set the same candidate bit"
        popc = [bin(int(x)).count("1") for x in f]
        wpre = np.concatenate([[0], np.cumsum(popc)]).astype(np.int64)
        new = []
        for row, key in best.items():  # k_dassign
            c = cand[row]
            below = (1 << (c & 31)) - 1
            sid = layer_end + int(wpre[c >> 5]) + bin(int(f[c >> 5]) & below).count("1")
            new.append((sid, np.frombuffer(row, np.uint64).copy(), key >> 32, key & 0xFFFFFFFF))
        new.sort(key=lambda x: x[0])
        for sid, row, _, _ in new:
            store[row.tobytes()] = sid
        lb_local = len(mine)
        mine.extend(new)
        N = int(wpre[-1])
        counts.append((E, G, N))
        n_total += N
        layer_begin, layer_end = layer_end, n_total
    return {"states": n_total, "layer_counts": counts, "local": mine}


def _protocol_worker(rank, world, port, cases, out, shard_from=1):
    _init(rank, world, port)
    try:
        for name, text, depth in cases:
            r = sharded_brfs_model(text, rank, world, depth, shard_from=shard_from)
            shards: list = [None] * world
            td.all_gather_object(shards, r["local"])
            if rank == 0:
                allst = sorted((s for sh in shards for s in sh), key=lambda x: x[0])
                out[name] = {
                    "states": r["states"],
                    "layer_counts": r["layer_counts"],
                    "ids": [s[0] for s in allst],
                    "rows": np.array([s[1] for s in allst], np.uint64),
                    "parent": [s[2] for s in allst],
                    "index": [s[3] for s in allst],
                    "sizes": [len(sh) for sh in shards],
                }
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("shard_from", [1, 40])
@pytest.mark.parametrize("world", [2, 3])
def test_sharded_protocol_matches_reference_ids(ref, world, shard_from):
    """Hash-owner sharding, global candidate indices and owner-side minimum discovery give the reference's ids; with
    shard_from 40 the small layers are replicated first and the ranks shard from the first frontier of 40 states."""
    from oracle import ref as oref

    cases = [("tower5", tasks.tower(5, 3), None), ("transport", tasks.transport(2, 6, 2, 0), None),
             ("tile3x3", tasks.sliding_tile(3, 3, 30, 0), 10),
             # the root has more than 255 successors: word lanes from the first layer on
             ("transport200", tasks.transport(2, 200, 3, 0), 2)]
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_protocol_worker, args=(world, _free_port(), cases, out, shard_from), nprocs=world,
                       join=True, start_method="spawn")
    for name, text, depth in cases:
        got = out[name]
        t = oref.RefTask(text)
        exp = t.brfs(max_depth=depth, stop_at_goal=False)
        rows, par, idx = t.brfs_states(max_depth=depth)
        assert got["states"] == exp["states"] == len(rows), name
        assert [tuple(x) for x in got["layer_counts"]] == exp["layer_counts"], name
        assert got["ids"] == list(range(len(rows))), name
        np.testing.assert_array_equal(got["rows"], rows, err_msg=name)
        assert got["parent"] == [int(x) for x in par], name
        assert got["index"] == [int(x) for x in idx], name
        assert min(got["sizes"]) > 0, f"{name}: a rank owns no state"
    assert out["transport200"]["layer_counts"][0][1] > 255


def _comm_id_worker(rank, world, port, out):
    _init(rank, world, port)
    try:
        out[rank] = bdist.broadcast_comm_id()
    finally:
        td.destroy_process_group()


def test_comm_id_broadcast_gloo():
    """Rank 0's NCCL id reaches every rank unchanged (the communicator set-up, without a GPU)."""
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_comm_id_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    assert len(out[0]) == 128 and out[0] == out[1]


def _membership_worker(rank, world, port, out):
    _init(rank, world, port)
    try:
        store = bdist.default_store()
        m = bdist.Membership(store, "b2comm/test", rank)
        m.check()  # everyone is in
        td.barrier()
        if rank == world - 1:
            m.leave()  # between searches: nothing of this rank is in flight
            m.leave()  # leaving twice counts once
            store.set("left-done", b"1")
            out[rank] = "left"
        else:
            store.wait(["left-done"])
            try:
                m.check()
                out[rank] = "not detected"
            except bdist.RankLeft as e:
                out[rank] = str(e)
        td.barrier()
    finally:
        td.destroy_process_group()


def test_rank_that_leaves_between_searches_is_detected_before_launch():
    """A rank that leaves the communicator between searches (Communicator.leave) is seen by the others on the host,
    through the process group's store, before their next search launches anything: the search raises RankLeft."""
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_membership_worker, args=(3, _free_port(), out), nprocs=3, join=True, start_method="spawn")
    assert out[2] == "left"
    for r in (0, 1):
        assert "1 rank(s) left" in out[r], out[r]


class _FakeResult:
    def __init__(self, shard):
        self.shard = shard

    def local(self, rows=True, hashes=True, nodes=True):
        return self.shard


def _gather_worker(rank, world, port, out):
    _init(rank, world, port)
    try:
        n = 37
        ids = np.array([i for i in range(n) if i % world == rank], np.uint64)
        shard = {"ids": ids, "rows": np.stack([ids, ids * 3], 1), "hashes": ids * 7,
                 "parent": (ids // 2).astype(np.uint32), "index": (ids % 5).astype(np.uint32)}
        g = bdist.gather_states(_FakeResult(shard))
        out[rank] = {k: v.tolist() for k, v in g.items()}
    finally:
        td.destroy_process_group()


def test_gather_states_gloo():
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_gather_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    for rank in (0, 1):
        g = out[rank]
        assert g["ids"] == list(range(37))
        assert g["rows"] == [[i, 3 * i] for i in range(37)]
        assert g["parent"] == [i // 2 for i in range(37)]


def test_merge_shards_rejects_bad_partitions():
    a = {"ids": np.array([0, 2], np.uint64)}
    b = {"ids": np.array([1, 2], np.uint64)}
    with pytest.raises(RuntimeError):
        bdist.merge_shards([a, b])
    c = {"ids": np.array([1, 3], np.uint64)}
    assert bdist.merge_shards([a, c])["ids"].tolist() == [0, 1, 2, 3]


def test_owner_partition_is_balanced():
    """The owner map spreads the hashes of a real state space evenly (every shard within 5 binomial standard
    deviations of its mean)."""
    from oracle import port as oport

    if not oport.available():
        pytest.skip("port oracle not built")
    t = oport.PortTask(tasks.sliding_tile(3, 3, 30, 0))
    r = t.brfs(max_depth=14, rows=True)
    hs = [oport.hash_row(row) for row in r["rows"]]
    for world in (2, 4, 8):
        sizes = np.bincount([owner_of(h, world) for h in hs], minlength=world)
        mean = len(hs) / world
        assert np.abs(sizes - mean).max() < 5 * np.sqrt(mean), (world, sizes)
