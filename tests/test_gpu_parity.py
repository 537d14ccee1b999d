"""Device path vs the reference's CPU path (oracle/_ref), bit for bit: BrFS states, ids, node records, per-layer
counts and fingerprints; batched expand CSR (labels and successor hashes); env trajectories; row hashes.

Mirrors the reference's device-vs-host tests (tests/cuda/test_device_brfs.cpp:131-360,
tests/cuda/test_device_env.cpp:254-460 in maichmueller/mymyr)."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from mymyr_b200 import cuda as b2cuda  # noqa: E402
from mymyr_b200 import rl as b2rl  # noqa: E402
from mymyr_b200 import tasks  # noqa: E402
from mymyr_b200.task import Task  # noqa: E402
from mymyr_b200 import UnsupportedTask  # noqa: E402


MATCHERS = ["compiled", "interpreted"]


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def random_states(task_words: int, slots: int, n: int, density: float, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    bits = rng.random((n, task_words * 64)) < density
    bits[:, slots:] = False
    out = np.zeros((n, task_words), np.uint64)
    for w in range(task_words):
        chunk = bits[:, w * 64:(w + 1) * 64].astype(np.uint64)
        out[:, w] = (chunk << np.arange(64, dtype=np.uint64)).sum(axis=1, dtype=np.uint64)
    return out


def to_dev(a: np.ndarray):
    return torch.from_numpy(a.view(np.int64)).cuda()


def as_u64(t):
    return t.cpu().numpy().view(np.uint64)


# ------------------------------------------------------------------------------------------------ hashing

def test_hash_rows_match_reference(ref):
    for W in (1, 2, 3, 4, 7, 13):
        rows = np.random.default_rng(W).integers(0, 2**63, (257, W), dtype=np.int64).view(np.uint64)
        rows[::3, W // 2:] = 0  # trimmed widths
        rows[5] = 0
        got = as_u64(b2cuda.hash_rows(to_dev(rows)))
        want = np.array([ref.hash_state(r) for r in rows], np.uint64)
        assert np.array_equal(got, want)


def test_hash_rows_numeric_words_match_reference(ref):
    # rows [atom words | numeric words]: the numeric words seed the hash of the trimmed atom words
    for W, nnum in ((2, 1), (3, 1), (4, 2), (7, 3), (5, 5)):
        rows = np.random.default_rng(W * 10 + nnum).integers(0, 2**63, (129, W), dtype=np.int64).view(np.uint64)
        rows[::3, : W - nnum][:, (W - nnum) // 2:] = 0  # trimmed atom widths
        rows[4, W - nnum:] = 0  # zero numeric words still seed
        got = as_u64(b2cuda.hash_rows(to_dev(rows), numeric_words=nnum))
        want = np.array([ref.hash_state(r, nnum) for r in rows], np.uint64)
        assert np.array_equal(got, want)
        assert np.array_equal(as_u64(b2cuda.hash_rows(to_dev(rows), numeric_words=0)),
                              np.array([ref.hash_state(r) for r in rows], np.uint64))


# ------------------------------------------------------------------------------------------------ BrFS

BRFS_CASES = [
    ("tower7", lambda: tasks.tower(7, 0), None),
    ("tower5_seed3", lambda: tasks.tower(5, 3), None),
    ("transport_2_6_2", lambda: tasks.transport(2, 6, 2, 1), None),
    ("transport_3_4_1", lambda: tasks.transport(3, 4, 1, 2), None),
    ("tile3x3", lambda: tasks.sliding_tile(3, 3, 40, 5), None),
    ("tile4x4_d12", lambda: tasks.sliding_tile(4, 4, 60, 0), 12),
    ("counters", lambda: tasks.counters(4, 6, 1), None),
    # witness-only parameters before effect parameters: under witness pruning the bindings are emitted sorted
    ("random600_d2", lambda: tasks.random_domain(0, n_init=600), 2),
]


@pytest.mark.parametrize("name,make,depth", BRFS_CASES, ids=[c[0] for c in BRFS_CASES])
@pytest.mark.parametrize("witness", [True, False])
@pytest.mark.parametrize("matcher", MATCHERS)
def test_brfs_matches_reference(ref, name, make, depth, witness, matcher):
    text = make()
    rt = ref.RefTask(text)
    t = Task.from_text(text, matcher=matcher)
    want = rt.brfs(threads=1, max_depth=depth, stop_at_goal=False, witness_pruning=witness, fingerprint=True)
    got = b2cuda.brfs(t, max_depth=depth, stop_at_goal=False, witness_pruning=witness, fingerprint=True)
    assert got.states == want["states"]
    assert got.expanded == want["expanded"]
    assert got.generated == want["generated"]
    assert got.num_goal_states == want["num_goal_states"]
    assert got.layers == want["layers"]
    assert got.layer_counts == want["layer_counts"]
    assert got.exhausted == bool(want["exhausted"])
    assert got.solved == bool(want["solved"])
    assert got.fingerprint == want["fingerprint"]
    # the stored states, ids and node records, in id order
    rows, par, idx = rt.brfs_states(max_depth=depth, witness_pruning=witness)
    assert np.array_equal(got.state_rows(), rows)
    p, k = got.nodes()
    assert np.array_equal(p, par)
    assert np.array_equal(k, idx)
    hs = got.state_hashes()
    assert len(hs) == len(rows)
    assert np.array_equal(hs[:500], np.array([ref.hash_state(r) for r in rows[:500]], np.uint64))


@pytest.mark.parametrize("make", [lambda: tasks.tower(7, 0), lambda: tasks.sliding_tile(3, 3, 30, 1),
                                  lambda: tasks.transport(2, 5, 2, 4)])
@pytest.mark.parametrize("matcher", MATCHERS)
def test_brfs_stop_at_goal_matches_reference(ref, make, matcher):
    text = make()
    rt = ref.RefTask(text)
    want = rt.brfs(threads=1, stop_at_goal=True, fingerprint=True)
    got = b2cuda.brfs(Task.from_text(text, matcher=matcher), stop_at_goal=True, fingerprint=True)
    for key in ("states", "expanded", "generated", "num_goal_states", "layers", "fingerprint"):
        assert getattr(got, key) == want[key], key
    assert got.solved == bool(want["solved"])
    assert got.layer_counts == want["layer_counts"]


@pytest.mark.parametrize("name,make,depth", BRFS_CASES, ids=[c[0] for c in BRFS_CASES])
@pytest.mark.parametrize("witness", [True, False])
@pytest.mark.parametrize("presize", ["exact", "small"])
def test_brfs_device_loop_matches_reference(ref, name, make, depth, witness, presize):
    """The layer loop as one CUDA graph launch (compiled matcher, buffers presized by expected_states, no per-layer
    events): the reference's states, ids and node records; with buffers too small for the later layers the search
    continues in the host loop from the layer that did not fit."""
    text = make()
    rt = ref.RefTask(text)
    t = Task.from_text(text, matcher="compiled")
    want = rt.brfs(threads=1, max_depth=depth, stop_at_goal=False, witness_pruning=witness, fingerprint=True)
    expected = want["states"] if presize == "exact" else 64
    got = b2cuda.brfs(t, max_depth=depth, stop_at_goal=False, witness_pruning=witness, fingerprint=True,
                      expected_states=expected)
    for key in ("states", "expanded", "generated", "num_goal_states", "layers", "fingerprint"):
        assert getattr(got, key) == want[key], key
    assert got.layer_counts == want["layer_counts"]
    assert got.exhausted == bool(want["exhausted"]) and got.solved == bool(want["solved"])
    rows, par, idx = rt.brfs_states(max_depth=depth, witness_pruning=witness)
    assert np.array_equal(got.state_rows(), rows)
    p, k = got.nodes()
    assert np.array_equal(p, par) and np.array_equal(k, idx)


@pytest.mark.parametrize("make", [lambda: tasks.tower(7, 0), lambda: tasks.sliding_tile(3, 3, 30, 1),
                                  lambda: tasks.transport(2, 5, 2, 4)])
def test_brfs_device_loop_stop_at_goal(ref, make):
    text = make()
    rt = ref.RefTask(text)
    want = rt.brfs(threads=1, stop_at_goal=True, fingerprint=True)
    t = Task.from_text(text, matcher="compiled")
    got = b2cuda.brfs(t, stop_at_goal=True, fingerprint=True, expected_states=want["states"] + 1000)
    for key in ("states", "expanded", "generated", "num_goal_states", "layers", "fingerprint"):
        assert getattr(got, key) == want[key], key
    assert got.solved == bool(want["solved"])
    assert got.layer_counts == want["layer_counts"]
    assert got.goal_id == b2cuda.brfs(t, stop_at_goal=True).goal_id  # the host loop's first goal state


def test_brfs_deterministic_across_runs():
    t = Task.from_text(tasks.sliding_tile(4, 4, 60, 7))
    a = b2cuda.brfs(t, max_depth=13, stop_at_goal=False, fingerprint=True)
    b = b2cuda.brfs(t, max_depth=13, stop_at_goal=False, fingerprint=True, expected_states=1 << 20)
    assert a.fingerprint == b.fingerprint and a.layer_counts == b.layer_counts
    assert b.stats.rehashes == 0 and a.stats.rehashes > 0  # growth does not change ids


@pytest.mark.slow
def test_brfs_tile_depth22_full_config(ref):
    """The 4x4 sliding-tile BrFS to depth 22 at full size: per-layer counts and fingerprint against the reference's multi-threaded BrFS
    (deterministic ids)."""
    import os

    text = tasks.sliding_tile(4, 4, 60, 0)
    want = ref.RefTask(text).brfs(threads=os.cpu_count() or 8, max_depth=22, stop_at_goal=False, fingerprint=True,
                                  store="concurrent")
    got = b2cuda.brfs(Task.from_text(text), max_depth=22, stop_at_goal=False, fingerprint=True)
    assert got.layer_counts == want["layer_counts"]
    assert got.states == want["states"] and got.generated == want["generated"]
    assert got.fingerprint == want["fingerprint"]
    # the device-driven layer loop (the bench's timed searches run this way)
    got = b2cuda.brfs(Task.from_text(text), max_depth=22, stop_at_goal=False, fingerprint=True,
                      expected_states=want["states"])
    assert got.layer_counts == want["layer_counts"] and got.fingerprint == want["fingerprint"]


# ------------------------------------------------------------------------------------------------ expand

EXPAND_CASES = [
    ("random", lambda: tasks.random_domain(0), 1024, 0.05),
    ("random_seed1", lambda: tasks.random_domain(1), 512, 0.08),
    ("tower7", lambda: tasks.tower(7, 0), 2048, 0.2),
    ("transport", lambda: tasks.transport(2, 40, 2, 0), 2048, 0.3),
    ("tile4x4", lambda: tasks.sliding_tile(4, 4, 60, 0), 2048, 0.1),
    ("counters", lambda: tasks.counters(4, 6, 1), 2048, 0.3),
]


@pytest.mark.parametrize("name,make,n,density", EXPAND_CASES, ids=[c[0] for c in EXPAND_CASES])
@pytest.mark.parametrize("witness", [False, True])
@pytest.mark.parametrize("matcher", MATCHERS)
def test_expand_matches_reference(ref, name, make, n, density, witness, matcher):
    text = make()
    rt = ref.RefTask(text)
    t = Task.from_text(text, matcher=matcher)
    states = random_states(t.words, t.fluent_slots, n, density, seed=hash(name) & 0xFFFF)
    states[0] = t.initial_state()
    want = rt.expand(states, witness_pruning=witness, succ=True)
    # the random domains' schemas bind witness-only parameters before effect parameters: under witness pruning their
    # bindings come out of the matcher out of canonical order and are emitted sorted
    got = b2rl.expand(t, to_dev(states), witness_pruning=witness, succ=True)
    assert got.generated == want["generated"]
    assert np.array_equal(got.offsets.cpu().numpy(), want["offsets"])
    assert np.array_equal(got.parent.cpu().numpy(), want["parent"])
    assert np.array_equal(got.schema.cpu().numpy(), want["schema"])
    lw = want["binding"].shape[1]
    assert np.array_equal(got.binding.cpu().numpy()[:, :lw], want["binding"])
    assert np.array_equal(as_u64(got.succ_hash), want["succ_hash"])
    assert np.array_equal(as_u64(got.succ), want["succ"])


@pytest.mark.parametrize("matcher", MATCHERS)
def test_expand_full_stress_batch_matches_reference(ref, matcher):
    """The lifted successor-generation stress workload at its full size: 1,048,576 states of the seeded random domain
    (24 predicates, 16 schemas of 3-5 parameters, 200 typed objects) with every slot set at 5 % density, witness
    pruning off, canonical order. Offsets, parents, schemas, bindings and successor hashes equal the reference's
    rl::expand (its thread-pool overload) element for element; successor rows are compared on the first 8,192
    states."""
    import os

    text = tasks.random_domain(0)
    t = Task.from_text(text, matcher=matcher)
    n = 1 << 20
    states = tasks.bernoulli_rows(n, t.words, t.fluent_slots, 0.05, seed=0, device="cuda")
    host = states.cpu().numpy().view(np.uint64)
    rt = ref.RefTask(text)
    got = b2rl.expand(t, states, witness_pruning=False)
    want = rt.expand(host, witness_pruning=False, threads=max(1, min(32, os.cpu_count() or 1)))
    assert got.generated == want["generated"] > 5 * n
    assert np.array_equal(got.offsets.cpu().numpy(), want["offsets"])
    assert np.array_equal(got.parent.cpu().numpy(), want["parent"])
    assert np.array_equal(got.schema.cpu().numpy(), want["schema"])
    lw = want["binding"].shape[1]
    assert np.array_equal(got.binding.cpu().numpy()[:, :lw], want["binding"])
    assert np.array_equal(as_u64(got.succ_hash), want["succ_hash"])
    k = 8192
    part = b2rl.expand(t, states[:k].contiguous(), witness_pruning=False, succ=True)
    want_k = rt.expand(host[:k], witness_pruning=False, succ=True)
    assert np.array_equal(as_u64(part.succ), want_k["succ"])
    assert np.array_equal(as_u64(part.succ_hash), want_k["succ_hash"])


def test_expand_empty_batch():
    t = Task.from_text(tasks.tower(4, 0))
    e = b2rl.expand(t, torch.zeros((0, t.words), dtype=torch.int64, device="cuda"))
    assert e.generated == 0 and e.offsets.tolist() == [0]


# ------------------------------------------------------------------------------------------------ env

def _compare_env(env, renv):
    assert np.array_equal(as_u64(env.states), renv.states)
    assert np.array_equal(env.steps.cpu().numpy(), renv.steps)
    assert np.array_equal(as_u64(env.draws), renv.draws)
    assert np.array_equal(env.at_goal.cpu().numpy(), renv.at_goal)
    assert np.array_equal(env.count.cpu().numpy(), renv.count)


ENV_CASES = [
    ("transport", lambda: tasks.transport(2, 40, 2, 0), dict()),
    ("transport_small_trunc", lambda: tasks.transport(2, 3, 2, 1), dict(max_steps=17, step_reward=-0.5)),
    ("tower5", lambda: tasks.tower(5, 2), dict(goal_reward=2.5)),
    ("tile3x3", lambda: tasks.sliding_tile(3, 3, 10, 3), dict(max_steps=40)),
]


@pytest.mark.parametrize("name,make,cfg", ENV_CASES, ids=[c[0] for c in ENV_CASES])
@pytest.mark.parametrize("matcher", MATCHERS)
def test_env_trajectories_match_reference(ref, name, make, cfg, matcher):
    text = make()
    rt = ref.RefTask(text)
    t = Task.from_text(text, matcher=matcher)
    n, steps = 512, 120
    env = b2rl.BatchedEnv(t, n, seed=1234, first_env=7, **cfg)
    renv = ref.RefEnv(rt, n, seed=1234, first_env=7, **cfg)
    env.reset()
    renv.reset()
    _compare_env(env, renv)
    lw = renv.lw
    for s in range(steps):
        env.step()
        renv.step()
        torch.cuda.synchronize()
        _compare_env(env, renv)
        assert np.array_equal(env.reward.cpu().numpy(), renv.reward), s
        assert np.array_equal(env.terminated.cpu().numpy(), renv.terminated), s
        assert np.array_equal(env.truncated.cpu().numpy(), renv.truncated), s
        assert np.array_equal(env.goal.cpu().numpy(), renv.goal), s
        assert np.array_equal(env.invalid.cpu().numpy(), renv.invalid), s
        assert np.array_equal(env.schema.cpu().numpy(), renv.schema), s
        assert np.array_equal(env.binding.cpu().numpy()[:, :lw], renv.binding), s
        assert np.array_equal(as_u64(env.final_states), renv.final_states), s


@pytest.mark.parametrize("matcher", MATCHERS)
def test_env_given_actions_match_reference(ref, matcher):
    text = tasks.transport(2, 4, 2, 3)
    rt = ref.RefTask(text)
    t = Task.from_text(text, matcher=matcher)
    n = 300
    env = b2rl.BatchedEnv(t, n, seed=5)
    renv = ref.RefEnv(rt, n, seed=5)
    env.reset()
    renv.reset()
    rng = np.random.default_rng(0)
    for s in range(60):
        a = rng.integers(-2, 12, n).astype(np.int64)  # out-of-range indices are invalid moves
        env.step(torch.from_numpy(a).cuda())
        renv.step(a)
        _compare_env(env, renv)
        assert np.array_equal(env.invalid.cpu().numpy(), renv.invalid)
        assert np.array_equal(env.reward.cpu().numpy(), renv.reward)


def test_env_next_task_ids(ref):
    """next_task_ids of a one-task env: ids of 0 change nothing; another id is reported once by check_errors
    (ValueError) and the rows keep their task, so the trajectories still equal the reference's."""
    text = tasks.transport(2, 4, 2, 3)
    rt = ref.RefTask(text)
    t = Task.from_text(text)
    n = 256
    env = b2rl.BatchedEnv(t, n, seed=9, max_steps=7)
    renv = ref.RefEnv(rt, n, seed=9, max_steps=7)
    env.reset()
    renv.reset()
    zeros = torch.zeros(n, dtype=torch.int32, device="cuda")
    bad = zeros.clone()
    bad[17] = 3
    for s in range(30):
        env.step(next_task_ids=bad if s == 11 else zeros)
        renv.step()
        _compare_env(env, renv)
        assert np.array_equal(env.reward.cpu().numpy(), renv.reward), s
        if s == 11:
            with pytest.raises(ValueError, match="next_task_ids"):
                env.check_errors()
        else:
            env.check_errors()
    with pytest.raises(ValueError):
        env.step(next_task_ids=zeros[:5])


def _step_digest(reward, terminated, truncated, goal, schema, count, binding):
    """One step's outputs of every env folded into a few integers (row-weighted sums, exact in int64)."""
    w = np.arange(1, len(count) + 1, dtype=np.int64)
    return (int((reward.view(np.int32).astype(np.int64) * w).sum()), int((terminated.astype(np.int64) * w).sum()),
            int((truncated.astype(np.int64) * w).sum()), int((goal.astype(np.int64) * w).sum()),
            int((schema.astype(np.int64) * w).sum()), int((count.astype(np.int64) * w).sum()),
            int((binding.astype(np.int64) * w[:, None]).sum()))


@pytest.mark.slow
def test_env_full_config_digest(ref):
    """The batched env step at its full size: 65,536 envs of the two-room transport task (40 balls, 2 grippers), random
    policy, seed 0, autoreset, for all 1,000 steps. Every step's outputs (rewards, terminated, truncated, goal, chosen
    schema and binding, successor counts) agree with the reference's HostEnv through a row-weighted digest, and the
    full state rows and counters are compared every 100 steps and after the last."""
    import os

    text = tasks.transport(2, 40, 2, 0)
    rt = ref.RefTask(text)
    t = Task.from_text(text)
    n, steps = 65536, 1000
    env = b2rl.BatchedEnv(t, n, seed=0)
    renv = ref.RefEnv(rt, n, seed=0, threads=max(1, min(64, os.cpu_count() or 8)))
    env.reset()
    renv.reset()
    lw = renv.lw
    for s in range(steps):
        env.step()
        renv.step()
        got = _step_digest(env.reward.cpu().numpy(), env.terminated.cpu().numpy(), env.truncated.cpu().numpy(),
                           env.goal.cpu().numpy(), env.schema.cpu().numpy(), env.count.cpu().numpy(),
                           env.binding.cpu().numpy()[:, :lw])
        want = _step_digest(renv.reward, renv.terminated, renv.truncated, renv.goal, renv.schema, renv.count,
                            renv.binding)
        assert got == want, s
        if (s + 1) % 100 == 0:
            _compare_env(env, renv)


MAX_STATES_CASES = [
    ("tower5", lambda: tasks.tower(5, 3), None),
    ("tile3x3_d14", lambda: tasks.sliding_tile(3, 3, 30, 0), 14),
    ("transport_2_4_2", lambda: tasks.transport(2, 4, 2, 1), None),
]

REF_STATUS = {0: "solved", 1: "exhausted", 2: "out_of_states", 6: "unsolvable"}


@pytest.mark.parametrize("name,make,depth", MAX_STATES_CASES, ids=[c[0] for c in MAX_STATES_CASES])
@pytest.mark.parametrize("matcher", MATCHERS)
@pytest.mark.parametrize("stop", [False, True])
def test_brfs_max_states_matches_reference(ref, name, make, depth, matcher, stop):
    """max_states stops the search right after that many states are stored, inside the expansion that stores the
    last one (run_flat): states, expanded, generated, per-layer counts, goal count, status, fingerprint and the kept
    states' rows and node records equal the reference's."""
    text = make()
    rt = ref.RefTask(text)
    t = Task.from_text(text, matcher=matcher)
    full = rt.brfs(max_depth=depth, stop_at_goal=False)
    rows, par, idx = rt.brfs_states(max_depth=depth)
    n = full["states"]
    for M in sorted({1, 2, 3, 7, n // 3, n // 2 + 1, n - 1, n, n + 3}):
        exp = rt.brfs_limited(M, max_depth=depth, stop_at_goal=stop, fingerprint=True)
        r = b2cuda.brfs(t, max_states=M, max_depth=depth, stop_at_goal=stop, fingerprint=True)
        got = (r.states, r.expanded, r.generated, r.num_goal_states, r.layers, r.layer_counts, r.status,
               r.fingerprint)
        want = (exp["states"], exp["expanded"], exp["generated"], exp["num_goal_states"], exp["layers"],
                exp["layer_counts"], REF_STATUS[exp["status"]], exp["fingerprint"])
        assert got == want, (M, got, want)
        k = r.states
        np.testing.assert_array_equal(r.state_rows(), rows[:k])
        p, i = r.nodes()
        np.testing.assert_array_equal(p, par[:k])
        np.testing.assert_array_equal(i, idx[:k])
        r.close()


SHIM_CASES = [
    ("tower7", lambda: tasks.tower(7, 0), None, False),
    ("tile3x3_goal", lambda: tasks.sliding_tile(3, 3, 30, 1), None, True),
    ("tile4x4_d14", lambda: tasks.sliding_tile(4, 4, 60, 0), 14, False),
    ("transport_2_6_2", lambda: tasks.transport(2, 6, 2, 1), None, False),
]


@pytest.mark.parametrize("atoms", ["auto", "dense"])
@pytest.mark.parametrize("name,make,depth,stop", SHIM_CASES, ids=[c[0] for c in SHIM_CASES])
def test_reference_side_shim_brfs_matches_reference(ref, name, make, depth, stop, atoms):
    """mymyr::brfs and the shim's device brfs (include/mymyr_b200_shim.hpp: the same signature, options and result
    struct) on the same reference Task, default Auto atom slots included: states, expanded, generated, goal states,
    layers, per-layer counts, fingerprint and status agree."""
    if not ref.shim_available():
        pytest.skip("oracle/_ref/libshim_check.so not built")
    rc, dev, want, msg = ref.shim_brfs(make(), atoms, max_depth=depth, stop_at_goal=stop)
    assert rc == 0, (msg, dev, want)
    assert dev == want
