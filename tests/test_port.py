"""Pins the CPU restatement oracle (oracle/port) before anything trusts it: against the reference's golden BrFS counts
(tests/cpp/support/suite.hpp:31-54 of maichmueller/mymyr), its Philox known answers, and the compiled reference
(oracle/_ref) on the generated benchmark tasks."""

import os
from pathlib import Path

import numpy as np
import pytest

from mymyr_b200 import tasks

# the reference checkout (read-only; present where the oracle is built, absent on GPU boxes)
REF_TASKS = Path(os.environ.get("MYMYR_REFERENCE", Path(__file__).resolve().parents[2] / "reference")) / "tests" / "data" / "tasks"


@pytest.fixture(scope="module")
def port():
    from oracle import port as p

    if not p.available():
        pytest.skip("port oracle not built (make -C oracle port)")
    return p


# exhaustive BrFS with witness pruning on: (states, generated, goal states)
GOLDEN = {
    "depot__p02": (40320, 376560, 9),
    "pegsol-08-strips__p22": (99457, 189967, 2),
    "gripper__prob05": (376832, 2031616, 2),
}


@pytest.mark.parametrize("name", ["depot__p02", "pegsol-08-strips__p22"])
def test_port_reproduces_suite_golden_counts(port, name):
    path = REF_TASKS / f"{name}.txt"
    if not path.exists():
        pytest.skip("reference fixtures absent")
    r = port.PortTask(path.read_text()).brfs()
    assert (r["states"], r["generated"], r["num_goal_states"]) == GOLDEN[name]


def test_port_philox_known_answer(port):
    # counter (draw lo, draw hi, env, purpose) = (0, 0, 0, 0), key (0, 0): Random123 vector 6627e8d5 e169c58d
    assert port.lib().port_philox_bits64(0, 0, 0) == 0xE169C58D6627E8D5


def test_port_hash_ignores_trailing_zero_words(port):
    a = np.array([0xDEADBEEF, 42, 0, 0], np.uint64)
    assert port.hash_row(a) == port.hash_row(a[:2])
    assert port.hash_row(np.zeros(3, np.uint64)) == port.hash_row(np.zeros(0, np.uint64))


CASES = {
    "tower6": lambda: tasks.tower(6, 1),
    "tower5_s3": lambda: tasks.tower(5, 3),
    "transport_2_4_2": lambda: tasks.transport(2, 4, 2, 1),
    "tile3x3": lambda: tasks.sliding_tile(3, 3, 30, 1),
}


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("witness", [True, False])
def test_port_brfs_matches_reference(port, ref, name, witness):
    text = CASES[name]()
    p = port.PortTask(text).brfs(witness_pruning=witness, rows=True)
    rt = ref.RefTask(text)
    r = rt.brfs(threads=1, stop_at_goal=False, witness_pruning=witness, fingerprint=True)
    for k in ("states", "expanded", "generated", "num_goal_states", "layers", "fingerprint"):
        assert p[k] == r[k], k
    assert p["layer_counts"] == r["layer_counts"]
    rows, _, _ = rt.brfs_states(witness_pruning=witness)
    assert np.array_equal(p["rows"], rows)


@pytest.mark.parametrize("name,make,n,density", [
    ("random0", lambda: tasks.random_domain(0), 64, 0.05),
    ("tile4x4", lambda: tasks.sliding_tile(4, 4, 60, 0), 256, 0.1),
    ("transport", lambda: tasks.transport(2, 40, 2, 0), 256, 0.3),
])
def test_port_expand_matches_reference(port, ref, name, make, n, density):
    text = make()
    pt = port.PortTask(text)
    rt = ref.RefTask(text)
    assert pt.words == rt.words and pt.fluent_slots == rt.fluent_slots
    rng = np.random.default_rng(3)
    bits = rng.random((n, pt.words * 64)) < density
    bits[:, pt.fluent_slots:] = False
    states = np.zeros((n, pt.words), np.uint64)
    for w in range(pt.words):
        states[:, w] = (bits[:, w * 64:(w + 1) * 64].astype(np.uint64) << np.arange(64, dtype=np.uint64)).sum(
            axis=1, dtype=np.uint64)
    a = pt.expand(states, label_width=rt.label_width)
    b = rt.expand(states)
    assert a["generated"] == b["generated"]
    assert np.array_equal(a["offsets"], b["offsets"])
    assert np.array_equal(a["schema"], b["schema"])
    assert np.array_equal(a["binding"], b["binding"])
    assert np.array_equal(a["succ_hash"], b["succ_hash"])


def test_port_env_matches_reference(port, ref):
    text = tasks.transport(2, 5, 2, 3)
    rows, steps = 64, 40
    st, rs = port.PortTask(text).env_run(rows, steps, seed=11, first_env=4)
    rt = ref.RefTask(text)
    env = ref.RefEnv(rt, rows, seed=11, first_env=4)
    env.reset()
    total = np.zeros(rows, np.float32)
    for _ in range(steps):
        env.step()
        total += env.reward
    assert np.array_equal(st, env.states)
    assert np.array_equal(rs, total)
