"""b2_expand_noalloc, the batched expand for callers that cannot allocate device memory while they run (processes that
hold the GPU's memory in their own allocator, latency-bound callers that cannot take cudaMalloc's synchronization).
Called through the C ABI and compared with b2_expand on the same batch, bit for bit (the outputs are integers), on two
calls in a row: the shared scratch keeps the previous call's contents, and the second call must not see them. One
case runs in a fresh process where b2_expand_noalloc is the first call on a new context (its set-up must already be
done by the context), and one runs a task without action schemas after a call that left data in the scratch.

This file is collected last on purpose: if it fails, a run that stops at the first failure has run every other test."""

import ctypes as C
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from mymyr_b200 import _lib, tasks  # noqa: E402
from mymyr_b200.task import Task  # noqa: E402


def _expansion(task, n, W, capacity, dev):
    lw = max(1, task.label_width)
    bufs = dict(succ=torch.zeros((capacity, W), dtype=torch.int64, device=dev),
                parent=torch.zeros(capacity, dtype=torch.int32, device=dev),
                schema=torch.zeros(capacity, dtype=torch.int32, device=dev),
                binding=torch.zeros((capacity, lw), dtype=torch.int32, device=dev),
                offsets=torch.zeros(n + 1, dtype=torch.int32, device=dev),
                succ_hash=torch.zeros(capacity, dtype=torch.int64, device=dev))
    e = _lib.Expansion()
    e.capacity, e.words, e.label_width = capacity, W, lw
    for k, t in bufs.items():
        setattr(e, k, t.data_ptr())
    return e, bufs


def _random_rows(task, n, density, rng):
    bits = rng.random((n, task.words * 64)) < density
    bits[:, task.fluent_slots:] = False
    rows = np.zeros((n, task.words), np.uint64)
    for w in range(task.words):
        rows[:, w] = (bits[:, w * 64:(w + 1) * 64].astype(np.uint64) << np.arange(64, dtype=np.uint64)).sum(
            axis=1, dtype=np.uint64)
    return rows


def _call(fn, task, states, capacity):
    n, W = states.shape
    e, bufs = _expansion(task, n, W, capacity, states.device)
    _lib.check(fn(task.handle, states.data_ptr(), n, W, 0, C.byref(e), None))
    torch.cuda.synchronize()
    return e.generated, {k: v.cpu().numpy() for k, v in bufs.items()}


@pytest.mark.parametrize("make,n,density", [(lambda: tasks.transport(2, 40, 2, 0), 3000, 0.3),
                                            (lambda: tasks.random_domain(0), 1500, 0.05)])
def test_expand_noalloc_matches_expand_twice(make, n, density):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = _lib.lib()
    task = Task.from_text(make())
    rng = np.random.default_rng(7)
    for call in range(2):
        rows = _random_rows(task, n, density, rng)
        states = torch.from_numpy(rows.view(np.int64)).cuda()
        g_ref, want = _call(L.b2_expand, task, states, 1 << 20)
        g_new, got = _call(L.b2_expand_noalloc, task, states, 1 << 20)
        assert g_new == g_ref > 0, call
        for k in want:
            if k == "offsets":
                assert np.array_equal(got[k], want[k]), (call, k)
            else:
                assert np.array_equal(got[k][:g_ref], want[k][:g_ref]), (call, k)


def test_expand_noalloc_refuses_batches_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = _lib.lib()
    task = Task.from_text(tasks.random_domain(0))  # 16 schemas: 2^18 segments are 16,384 states
    n = (1 << 18) // task.num_schemas + 1
    states = torch.zeros((n, task.words), dtype=torch.int64, device="cuda")
    e, _ = _expansion(task, n, task.words, 16, states.device)
    rc = L.b2_expand_noalloc(task.handle, states.data_ptr(), n, task.words, 0, C.byref(e), None)
    assert rc == _lib.B2_CAPACITY
    assert "segments" in _lib.last_error()


_FRESH = textwrap.dedent("""
    import sys
    sys.path.insert(0, sys.argv[1])
    sys.path.insert(0, sys.argv[2])
    import numpy as np
    import torch
    import test_zz_no_alloc as t
    from mymyr_b200 import _lib, tasks
    from mymyr_b200.task import Context, Task
    ctx = Context(0)  # a new context: b2_expand_noalloc's set-up happens here
    task = Task.from_text(tasks.transport(2, 40, 2, 0), ctx)
    L = _lib.lib()
    rng = np.random.default_rng(11)
    rows = [torch.from_numpy(t._random_rows(task, 2000, 0.3, rng).view(np.int64)).cuda() for _ in range(2)]
    first = [t._call(L.b2_expand_noalloc, task, r, 1 << 20) for r in rows]  # the first calls of the process
    for (g_new, got), r in zip(first, rows):
        g_ref, want = t._call(L.b2_expand, task, r, 1 << 20)
        assert g_new == g_ref > 0
        for k in want:
            n = len(want[k]) if k == "offsets" else g_ref
            assert np.array_equal(got[k][:n], want[k][:n]), k
    print("fresh ok", first[0][0], first[1][0])
""")


def test_expand_noalloc_first_call_of_a_fresh_process():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    here = Path(__file__).resolve().parent
    r = subprocess.run([sys.executable, "-c", _FRESH, str(here.parent), str(here)], capture_output=True, text=True,
                       timeout=600, env=dict(os.environ))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "fresh ok" in r.stdout


def test_expand_noalloc_task_without_schemas_after_a_full_call():
    """A task with no action schemas has no segments: every offset is 0, whatever the previous call left behind."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = _lib.lib()
    busy = Task.from_text(tasks.transport(2, 40, 2, 0))
    rng = np.random.default_rng(5)
    states = torch.from_numpy(_random_rows(busy, 3000, 0.3, rng).view(np.int64)).cuda()
    assert _call(L.b2_expand_noalloc, busy, states, 1 << 20)[0] > 0
    t = tasks.TaskText(n=3)
    p = t.pred("F", 1, "p")
    t.fluent_init.append((p, (0,)))
    t.goal.append((p, True, (1,)))
    empty = Task.from_text(t.text())
    assert empty.num_schemas == 0
    n = 500
    rows = torch.zeros((n, empty.words), dtype=torch.int64, device="cuda")
    rows[:, 0] = 1
    g, got = _call(L.b2_expand_noalloc, empty, rows, 16)
    assert g == 0
    assert np.array_equal(got["offsets"], np.zeros(n + 1, np.int32))
