"""The sharded BrFS (one process per GPU, NCCL) against the reference: the same states, ids, node records, hashes,
layer counts and fingerprint as the reference's CPU BrFS with deterministic ids, on both matcher backends. World 1 (a
communicator of one rank, every record pushed to itself through the same kernels) runs on any box; larger worlds are
skipped on a box with fewer GPUs."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

from mymyr_b200 import tasks

pytestmark = pytest.mark.gpu

CASES = [
    # name, text, max_depth, witness pruning, stop at goal
    ("tower5", tasks.tower(5, 3), None, True, False),
    ("transport_2_6_2", tasks.transport(2, 6, 2, 0), None, True, False),
    ("transport_2_6_2_nw", tasks.transport(2, 6, 2, 0), None, False, False),
    ("tile3x3", tasks.sliding_tile(3, 3, 30, 0), None, True, False),
    ("tile4x4_d12", tasks.sliding_tile(4, 4, 60, 0), 12, True, False),
    ("tower7_goal", tasks.tower(7, 0), None, True, True),
    ("tile3x3_goal", tasks.sliding_tile(3, 3, 30, 0), None, True, True),
    # the root has more than 255 successors: the count lanes widen to words from the first layer on
    ("transport_2_200_3_d2", tasks.transport(2, 200, 3, 0), 2, True, False),
]


# shard_from_states: 1 shards from the root (every layer exchanges), 64 runs the first layers on every rank alone and
# shards from the first frontier of 64 states, 0 is the default (2^20: these small searches run replicated to the end)
SHARD_FROM = (1, 64, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, matcher, out):
    import torch.distributed as td

    from mymyr_b200 import Context, Task, cuda
    from mymyr_b200 import dist as bdist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                          timeout=datetime.timedelta(seconds=120))
    try:
        ctx = Context(rank)
        comm = bdist.Communicator(ctx, timeout_s=60)
        for name, text, depth, witness, stop in CASES:
            task = Task.from_text(text, ctx, matcher=matcher)
            for sf in SHARD_FROM:
                r = cuda.brfs(task, comm=comm, max_depth=depth, stop_at_goal=stop, fingerprint=True,
                              witness_pruning=witness, shard_from_states=sf)
                g = bdist.gather_states(r)
                if rank == 0:
                    out[(name, sf)] = {"states": r.states, "expanded": r.expanded, "generated": r.generated,
                                       "layer_counts": r.layer_counts, "fingerprint": r.fingerprint,
                                       "solved": r.solved, "goal_id": r.goal_id,
                                       "num_goal_states": r.num_goal_states, "rows": g["rows"],
                                       "parent": g["parent"], "index": g["index"], "hashes": g["hashes"]}
                out[(name, sf, rank)] = (r.stats.local_states, r.stats.exchanged, r.states, r.fingerprint)
                r.close()
        comm.close()
        td.barrier()
    finally:
        td.destroy_process_group()


def _run(world, matcher):
    import torch.multiprocessing as mp

    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), matcher, out), nprocs=world, join=True,
                       start_method="spawn")
    return dict(out)


def _worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return sorted({1, 2, n}) if n >= 2 else [1, 2]


@pytest.mark.parametrize("matcher", ["compiled", "interpreted"])
@pytest.mark.parametrize("world", _worlds())
def test_sharded_brfs_matches_reference(ref, world, matcher):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import ref as oref

    out = _run(world, matcher)
    for name, text, depth, witness, stop in CASES:
        t = oref.RefTask(text)
        exp = t.brfs(max_depth=depth, stop_at_goal=stop, witness_pruning=witness, fingerprint=True)
        rows, par, idx = t.brfs_states(max_depth=depth, witness_pruning=witness)
        for sf in SHARD_FROM:
            got, what = out[(name, sf)], (name, sf)
            assert got["states"] == exp["states"], what
            assert got["layer_counts"] == exp["layer_counts"], what
            assert got["fingerprint"] == exp["fingerprint"], what
            assert bool(got["solved"]) == bool(exp["solved"]), what
            assert got["num_goal_states"] == exp["num_goal_states"], what
            per_rank = [out[(name, sf, r)] for r in range(world)]
            assert sum(p[0] for p in per_rank) == got["states"], what  # the shards partition the states
            assert len({(p[2], p[3]) for p in per_rank}) == 1, what    # every rank reports the same result
            if not stop:
                np.testing.assert_array_equal(got["rows"], rows, err_msg=str(what))
                np.testing.assert_array_equal(got["parent"], par, err_msg=str(what))
                np.testing.assert_array_equal(got["index"], idx, err_msg=str(what))
                assert [int(h) for h in got["hashes"]] == [oref.hash_state(r) for r in rows], what
                if world > 1 and sf == 1:
                    assert sum(p[1] for p in per_rank) > 0, what  # successors crossed between ranks


MAX_STATES_CASES = [
    ("tower5", tasks.tower(5, 3), None),
    ("tile3x3_d14", tasks.sliding_tile(3, 3, 30, 0), 14),
    ("transport_2_4_2", tasks.transport(2, 4, 2, 1), None),
]
REF_STATUS = {0: "solved", 1: "exhausted", 2: "out_of_states", 6: "unsolvable"}


def _max_states_worker(rank, world, port, limits, out):
    import torch.distributed as td

    from mymyr_b200 import Context, Task, cuda
    from mymyr_b200 import dist as bdist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                          timeout=datetime.timedelta(seconds=120))
    try:
        ctx = Context(rank)
        comm = bdist.Communicator(ctx, timeout_s=60)
        for name, text, depth in MAX_STATES_CASES:
            task = Task.from_text(text, ctx)
            for stop, M, sf in [(st, m, sf) for st in (False, True) for m in limits[name] for sf in (1, 16, 0)]:
                r = cuda.brfs(task, comm=comm, max_states=M, max_depth=depth, stop_at_goal=stop,
                              fingerprint=True, shard_from_states=sf)
                g = bdist.gather_states(r)
                if rank == 0:
                    out[(name, stop, M, sf)] = {
                        "got": (r.states, r.expanded, r.generated, r.num_goal_states, r.layers, r.layer_counts,
                                r.status, r.fingerprint),
                        "rows": g["rows"], "parent": g["parent"], "index": g["index"]}
                r.close()
        comm.close()
        td.barrier()
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("world", _worlds())
def test_sharded_brfs_max_states_matches_reference(ref, world):
    """max_states on the sharded search: the reference's cut inside the expansion that stores the last state (run_flat)
    -- counts, per-layer counts, goal count, status, fingerprint, and the kept states, ids and node records."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from oracle import ref as oref

    limits = {}
    for name, text, depth in MAX_STATES_CASES:
        n = oref.RefTask(text).brfs(max_depth=depth, stop_at_goal=False)["states"]
        limits[name] = sorted({1, 2, 3, 7, n // 3, n // 2 + 1, n - 1, n, n + 3})
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_max_states_worker, args=(world, _free_port(), limits, out), nprocs=world, join=True,
                       start_method="spawn")
    for name, text, depth in MAX_STATES_CASES:
        rt = oref.RefTask(text)
        rows, par, idx = rt.brfs_states(max_depth=depth)
        for stop in (False, True):
            for M in limits[name]:
                exp = rt.brfs_limited(M, max_depth=depth, stop_at_goal=stop, fingerprint=True)
                want = (exp["states"], exp["expanded"], exp["generated"], exp["num_goal_states"], exp["layers"],
                        exp["layer_counts"], REF_STATUS[exp["status"]], exp["fingerprint"])
                for sf in (1, 16, 0):
                    got = out[(name, stop, M, sf)]
                    assert got["got"] == want, (name, stop, M, sf, got["got"], want)
                    k = exp["states"]
                    np.testing.assert_array_equal(got["rows"], rows[:k], err_msg=f"{name} {M} {sf}")
                    np.testing.assert_array_equal(got["parent"], par[:k], err_msg=f"{name} {M} {sf}")
                    np.testing.assert_array_equal(got["index"], idx[:k], err_msg=f"{name} {M} {sf}")


ASTAR_CASES = [
    ("tower5", tasks.tower(5, 3)),
    ("tile3x3", tasks.sliding_tile(3, 3, 30, 0)),
    ("logistics_small", tasks.logistics(3, 3, 2, 1, 3, 5)),
    ("logistics_2pk", tasks.logistics(8, 4, 6, 2, 2, 0)),
]


def _astar_worker(rank, world, port, matcher, out):
    import torch.distributed as td

    from mymyr_b200 import Context, Task, cuda
    from mymyr_b200 import dist as bdist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                          timeout=datetime.timedelta(seconds=120))
    try:
        ctx = Context(rank)
        comm = bdist.Communicator(ctx, timeout_s=60)
        for name, text in ASTAR_CASES:
            task = Task.from_text(text, ctx, matcher=matcher)
            r = cuda.astar(task, comm=comm)
            out[(name, rank)] = (r.status, r.cost, r.expanded, r.generated, r.states)
            r.close()
        comm.close()
        td.barrier()
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("matcher", ["compiled", "interpreted"])
@pytest.mark.parametrize("world", _worlds())
def test_sharded_astar_optimal_cost(ref, world, matcher):
    """A* with its states partitioned by state-hash owner finds the reference's optimal cost; every rank reports the
    same result, and it expands exactly the states of the one-GPU search (the same f layers)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from mymyr_b200 import Task, cuda

    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_astar_worker, args=(world, _free_port(), matcher, out), nprocs=world, join=True,
                       start_method="spawn")
    for name, text in ASTAR_CASES:
        per_rank = [out[(name, r)] for r in range(world)]
        assert len(set(per_rank)) == 1, (name, per_rank)
        status, cost, expanded, generated, states = per_rank[0]
        exp = ref.RefTask(text).astar()
        assert status == "solved" and cost == exp["cost"], (name, cost, exp["cost"])
        one = cuda.astar(Task.from_text(text, matcher=matcher))
        assert (expanded, generated, states) == (one.expanded, one.generated, one.states), name
        one.close()


def _overflow_worker(rank, world, port, matcher, out):
    import torch.distributed as td

    from mymyr_b200 import Context, Task, cuda
    from mymyr_b200 import _lib
    from mymyr_b200 import dist as bdist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                          timeout=datetime.timedelta(seconds=120))
    try:
        ctx = Context(rank)
        comm = bdist.Communicator(ctx, timeout_s=60)
        task = Task.from_text(tasks.sliding_tile(3, 3, 30, 0), ctx, matcher=matcher)
        try:
            cuda.brfs(task, comm=comm, stop_at_goal=False, max_exchange_records=40, shard_from_states=1)
            out[("small", rank)] = "ran"
        except _lib.CapacityError as e:
            out[("small", rank)] = "capacity: " + str(e)
        # the context and the communicator stay usable: the same search with room for its records
        r = cuda.brfs(task, comm=comm, stop_at_goal=False, fingerprint=True)
        out[("full", rank)] = (r.states, r.fingerprint, r.layer_counts)
        r.close()
        comm.close()
        td.barrier()
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("matcher", ["compiled", "interpreted"])
@pytest.mark.parametrize("world", _worlds())
def test_sharded_brfs_receive_buffer_overflow_fails_every_rank(ref, world, matcher):
    """A layer whose records do not fit a rank's receive buffer (bounded here by max_exchange_records) fails with
    B2_CAPACITY on every rank: the push kernels drop the records past the buffer instead of writing into another GPU's
    memory, and the next search on the same communicator runs normally."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_overflow_worker, args=(world, _free_port(), matcher, out), nprocs=world, join=True,
                       start_method="spawn")
    exp = ref.RefTask(tasks.sliding_tile(3, 3, 30, 0)).brfs(stop_at_goal=False, fingerprint=True)
    for r in range(world):
        assert out[("small", r)].startswith("capacity:"), out[("small", r)]
        assert "receive buffer" in out[("small", r)]
        states, fp, lc = out[("full", r)]
        assert (states, fp, lc) == (exp["states"], exp["fingerprint"], exp["layer_counts"])


def _leave_worker(rank, world, port, out):
    import torch.distributed as td

    from mymyr_b200 import Context, Task, cuda
    from mymyr_b200 import dist as bdist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast object outlives a rank that leaves
    torch.cuda.set_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                          timeout=datetime.timedelta(seconds=60))
    try:
        ctx = Context(rank)
        comm = bdist.Communicator(ctx, timeout_s=30)
        store = bdist.default_store()
        task = Task.from_text(tasks.sliding_tile(3, 3, 30, 0), ctx)
        r = cuda.brfs(task, comm=comm, stop_at_goal=False)
        out[("first", rank)] = r.states
        r.close()
        if rank == world - 1:
            comm.leave()  # between searches: none of its kernels or collectives is in flight
            store.set("b2-test-left", b"1")
        else:
            store.wait(["b2-test-left"])
            try:
                cuda.brfs(task, comm=comm, stop_at_goal=False)
                out[("second", rank)] = "ran"
            except bdist.RankLeft as e:
                out[("second", rank)] = "left: " + str(e)
            store.set("b2-test-checked", b"1")
        store.wait(["b2-test-checked"])
        comm.close()  # the communicator's teardown is collective: every rank, after the check
        td.barrier()
    finally:
        td.destroy_process_group()


def test_rank_leaving_between_searches_fails_the_others_on_the_host(ref):
    """A rank that leaves the communicator between searches: the other ranks' next search raises RankLeft on the host
    before it launches a kernel or a collective, so that no rank waits in a collective for a rank that is gone."""
    world = 2
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_leave_worker, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    exp = ref.RefTask(tasks.sliding_tile(3, 3, 30, 0)).brfs(stop_at_goal=False)
    assert out[("first", 0)] == out[("first", 1)] == exp["states"]
    assert out[("second", 0)].startswith("left: "), out[("second", 0)]
