"""b2_expand_noalloc, the batched expand for callers that cannot allocate device memory while they run (processes that
hold the GPU's memory in their own allocator, latency-bound callers that cannot take cudaMalloc's synchronization).
Called through the C ABI and compared with b2_expand on the same batch, bit for bit (the outputs are integers), on two
calls in a row: the shared scratch keeps the previous call's contents, and the second call must not see them.

This file is collected last on purpose: if it fails, a run that stops at the first failure has run every other test."""

import ctypes as C

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
        bits = rng.random((n, task.words * 64)) < density
        bits[:, task.fluent_slots:] = False
        rows = np.zeros((n, task.words), np.uint64)
        for w in range(task.words):
            rows[:, w] = (bits[:, w * 64:(w + 1) * 64].astype(np.uint64) << np.arange(64, dtype=np.uint64)).sum(
                axis=1, dtype=np.uint64)
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
