"""The host grounding of the delete relaxation (relax.cpp, behind h^max) against the reference's own grounding
(heuristics::ground, GroundingStats): the same reached atoms and the same ground actions on every task; and the
A*/h^max config's generator pinned by digest."""

from __future__ import annotations

import hashlib

import pytest

from mymyr_b200 import tasks
from mymyr_b200 import _lib
from mymyr_b200._lib import check, lib
from mymyr_b200.task import Task

import ctypes as C

CASES = {
    "tower5": lambda: tasks.tower(5, 3),
    "tower7": lambda: tasks.tower(7, 0),
    "transport_2_6_2": lambda: tasks.transport(2, 6, 2, 0),
    "tile3x3": lambda: tasks.sliding_tile(3, 3, 30, 0),
    "tile4x4": lambda: tasks.sliding_tile(4, 4, 60, 0),
    "logistics_2pk": lambda: tasks.logistics(8, 4, 6, 2, 2, 0),
    "logistics_30pk": lambda: tasks.logistics(8, 4, 6, 2, 30, 0),
    "logistics_small": lambda: tasks.logistics(3, 3, 2, 1, 3, 5),
}


def host_grounding(text: str) -> dict:
    t = Task.from_text(text, host_only=True)
    h = C.c_void_p()
    check(lib().b2_heuristic_create(t.handle, _lib.B2_HEURISTIC_MAX, C.byref(h)))
    info = _lib.HeuristicInfo()
    check(lib().b2_heuristic_info_get(h, C.byref(info)))
    lib().b2_heuristic_destroy(h)
    return {k: getattr(info, k) for k, _ in _lib.HeuristicInfo._fields_}


@pytest.mark.parametrize("name", sorted(CASES))
def test_grounding_matches_reference(ref, name):
    text = CASES[name]()
    got = host_grounding(text)
    exp = ref.RefTask(text).ground_stats()
    assert got["reached_atoms"] == exp["reached_atoms"], (got, exp)
    assert got["ground_actions"] == exp["ground_actions"], (got, exp)
    assert got["ops"] <= exp["operators"]  # operators that add nothing new are dropped here
    assert not got["goal_unreachable"]


def test_logistics_generator_digest():
    """The config's text is fixed by its seed (parity depends only on the emitted text)."""
    d = hashlib.sha256(tasks.logistics(8, 4, 6, 2, 2, 0).encode()).hexdigest()[:16]
    d30 = hashlib.sha256(tasks.logistics(8, 4, 6, 2, 30, 0).encode()).hexdigest()[:16]
    assert (d, d30) == (DIGEST_2, DIGEST_30)


DIGEST_2 = "892c8d50057e0648"
DIGEST_30 = "fd55c889f9945477"
