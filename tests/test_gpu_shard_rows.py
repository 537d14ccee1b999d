"""Row-sharded work (the env pool and the batched expand at N > 1 GPUs, one shard per rank) gives the results of the
whole batch: an env's trajectory depends only on its global env id (its RNG stream), and a state's successors only on
the state. Checked on one GPU by splitting a batch into shards."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mymyr_b200 import rl as b2rl
from mymyr_b200 import tasks
from mymyr_b200.task import Task

pytestmark = pytest.mark.gpu


def as_u64(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint64)


def test_env_shards_by_env_index():
    t = Task.from_text(tasks.transport(2, 6, 2, 1))
    n, cut, steps = 1000, 600, 80
    whole = b2rl.BatchedEnv(t, n, seed=77, max_steps=30)
    parts = [b2rl.BatchedEnv(t, cut, seed=77, max_steps=30, first_env=0),
             b2rl.BatchedEnv(t, n - cut, seed=77, max_steps=30, first_env=cut)]
    for e in [whole, *parts]:
        e.reset()
    for s in range(steps):
        whole.step()
        for e in parts:
            e.step()
        torch.cuda.synchronize()
        for name in ("states", "reward", "terminated", "truncated", "count", "schema", "binding"):
            got = torch.cat([getattr(e, name) for e in parts]).cpu().numpy()
            assert np.array_equal(getattr(whole, name).cpu().numpy(), got), (s, name)


def test_expand_shards_by_row():
    t = Task.from_text(tasks.random_domain(1))
    rng = np.random.default_rng(3)
    n, cut, W = 700, 300, t.words
    rows = np.zeros((n, W), np.uint64)
    bits = rng.random((n, t.fluent_slots)) < 0.05
    for i, j in zip(*np.nonzero(bits)):
        rows[i, j >> 6] |= np.uint64(1) << np.uint64(j & 63)
    states = torch.from_numpy(rows.view(np.int64)).cuda()
    whole = b2rl.expand(t, states, witness_pruning=False)
    a = b2rl.expand(t, states[:cut], witness_pruning=False)
    b = b2rl.expand(t, states[cut:], witness_pruning=False)
    off = np.concatenate([a.offsets.cpu().numpy()[:-1], b.offsets.cpu().numpy() + int(a.offsets[-1])])
    assert np.array_equal(whole.offsets.cpu().numpy(), off)
    assert np.array_equal(whole.parent.cpu().numpy(),
                          np.concatenate([a.parent.cpu().numpy(), b.parent.cpu().numpy() + cut]))
    for name in ("schema", "binding", "succ_hash"):
        got = torch.cat([getattr(a, name), getattr(b, name)]).cpu().numpy()
        assert np.array_equal(getattr(whole, name).cpu().numpy(), got), name
