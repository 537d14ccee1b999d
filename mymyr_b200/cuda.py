"""Device searches: ``brfs`` mirrors mymyr.cuda.brfs (python/src/cuda_bindings.cpp:2715-2745 in maichmueller/mymyr) and
returns a result with the fields of BrfsResult and DeviceBrfsStats; ``astar`` mirrors mymyr.cuda.astar with h^max
(python/src/cuda_heuristics_bindings.cpp:518) and ``Heuristic`` mymyr.cuda.Heuristic's h^max (:385-450); ``hash_rows``
mirrors mymyr.hash_rows (python/src/module.cpp:187)."""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import check, lib
from .task import Context, Task

STATUS = {0: "solved", 1: "exhausted", 2: "out_of_states", 3: "unsolvable"}


@dataclass
class DeviceBrfsStats:
    """Per-phase device times (with timings=True) and table facts (cuda::DeviceBrfsStats)."""

    count_ms: float = 0.0
    gen_ms: float = 0.0
    dedup_ms: float = 0.0
    rehashes: int = 0
    table_slots: int = 0
    kernel_launches: int = 0
    local_states: int = 0  # states this rank stores (all of them on one GPU)
    exchanged: int = 0     # successors this rank received from other ranks (sharded search)
    exchange_ms: float = 0.0  # sharded search: device time of the successor exchange (part of gen_ms)
    wait_ms: float = 0.0      # host time spent waiting for the per-layer results (of search_s)


@dataclass
class BrfsResult:
    status: str
    states: int
    expanded: int
    generated: int
    num_goal_states: int
    layers: int
    layer_counts: list
    exhausted: bool
    solved: bool
    goal_id: int
    fingerprint: int
    search_s: float
    words: int
    stats: DeviceBrfsStats = field(default_factory=DeviceBrfsStats)
    store: str = "device"
    _search: object = None

    def state_rows(self, first: int = 0, count: int | None = None) -> np.ndarray:
        """State rows in id order (DeviceBrfs::states), [count, words] uint64."""
        return self._search.states(first, count)

    def nodes(self, first: int = 0, count: int | None = None):
        """Node records (parent id, successor index) of states [first, first + count) (DeviceBrfs::nodes)."""
        return self._search.nodes(first, count)

    def state_hashes(self, first: int = 0, count: int | None = None) -> np.ndarray:
        """hash::state of every stored state, in id order."""
        return self._search.hashes(first, count)

    def local(self, first: int = 0, count: int | None = None, *, rows: bool = True, hashes: bool = True,
              nodes: bool = True) -> dict:
        """The states this rank stores (all states on one GPU), in id order: ``ids`` and, as asked, ``rows``,
        ``hashes``, ``parent`` and ``index`` (numpy arrays). A sharded search's states are read this way, per rank;
        ``mymyr_b200.dist.gather_states`` assembles them over the ranks."""
        return self._search.local(first, count, rows=rows, hashes=hashes, nodes=nodes)

    def close(self) -> None:
        """Releases the device state space (state_rows, nodes and state_hashes are unavailable afterwards)."""
        if self._search is not None:
            self._search.close()
            self._search = None


class _Search:
    def __init__(self, task: Task, opts: _lib.BrfsOptions):
        self.task = task
        h = C.c_void_p()
        check(lib().b2_brfs_create(task.handle, C.byref(opts), C.byref(h)))
        self._h = h
        self.n = 0

    def run(self, layer_cap: int = 4096) -> _lib.BrfsResult:
        lc = np.zeros((layer_cap, 3), np.uint64)
        r = _lib.BrfsResult()
        r.layer_counts = lc.ctypes.data_as(C.POINTER(C.c_uint64))
        r.layer_capacity = layer_cap
        check(lib().b2_brfs_run(self._h, C.byref(r)))
        self.n = r.states
        self.lc = lc[: min(r.layers, layer_cap)]
        return r

    def _range(self, first, count):
        if count is None:
            count = self.n - first
        return first, count

    def states(self, first=0, count=None):
        first, count = self._range(first, count)
        out = np.zeros((count, self.task.words), np.uint64)
        check(lib().b2_brfs_states(self._h, first, count, out.ctypes.data, self.task.words))
        return out

    def nodes(self, first=0, count=None):
        first, count = self._range(first, count)
        p = np.zeros(count, np.uint32)
        k = np.zeros(count, np.uint32)
        check(lib().b2_brfs_nodes(self._h, first, count, p.ctypes.data, k.ctypes.data))
        return p, k

    def hashes(self, first=0, count=None):
        first, count = self._range(first, count)
        out = np.zeros(count, np.uint64)
        check(lib().b2_brfs_state_hashes(self._h, first, count, out.ctypes.data))
        return out

    def local(self, first=0, count=None, *, rows=True, hashes=True, nodes=True):
        n = C.c_uint64()
        check(lib().b2_brfs_local_count(self._h, C.byref(n)))
        if count is None:
            count = n.value - first
        out = {"ids": np.zeros(count, np.uint64)}
        if rows:
            out["rows"] = np.zeros((count, self.task.words), np.uint64)
        if hashes:
            out["hashes"] = np.zeros(count, np.uint64)
        if nodes:
            out["parent"] = np.zeros(count, np.uint32)
            out["index"] = np.zeros(count, np.uint32)
        ptr = lambda k: out[k].ctypes.data if k in out else None  # noqa: E731
        check(lib().b2_brfs_local(self._h, first, count, ptr("ids"), ptr("rows"), self.task.words, ptr("hashes"),
                                  ptr("parent"), ptr("index")))
        return out

    def close(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.b2_brfs_destroy(h)
        self._h = None

    def __del__(self):
        self.close()


def brfs(task: Task, *, ctx: Context | None = None, witness_pruning: bool = True, canonical_order: bool = True,
         max_states: int | None = None, stop_at_goal: bool = True, fingerprint: bool = False,
         chunk_states: int | None = None, expected_states: int | None = None, max_depth: int | None = None,
         timings: bool = False, stream=None, comm=None, max_exchange_records: int | None = None,
         shard_from_states: int | None = None) -> BrfsResult:
    """The device BrFS (mymyr.cuda.brfs, python/src/cuda_bindings.cpp:2715-2771: the same keywords and defaults).
    Ids, per-layer counts and the fingerprint equal the reference CPU BrFS with deterministic ids.
    ``canonical_order=False`` leaves the successor order of a (state, schema) to the matcher in the reference; here
    the search runs in canonical order, one of the orders it allows. ``chunk_states`` is accepted for signature
    compatibility: layers are never chunked here, and ids do not depend on it. ``comm`` (a
    ``mymyr_b200.dist.Communicator``) shards the search over its ranks by state hash: every rank calls brfs together
    and gets the same result; each rank reads its own states with ``BrfsResult.local``. ``max_exchange_records``
    bounds the successor records a rank takes in per layer (a layer that needs more raises CapacityError on every
    rank, B2_CAPACITY). ``shard_from_states``: with ``comm``, every rank runs the layers alone (the same search, no
    exchange) until a frontier holds this many states (default 2^20; 1: shard from the root); the result does not
    depend on it."""
    if chunk_states is not None and int(chunk_states) < 1:
        raise ValueError("mymyr_b200 brfs: chunk_states must be at least 1")
    if ctx is not None and task.ctx is not None and ctx.device != task.ctx.device:
        raise ValueError("mymyr_b200 brfs: the task lives on another device than ctx")
    o = _lib.BrfsOptions()
    lib().b2_brfs_options_default(C.byref(o))
    o.witness_pruning = int(bool(witness_pruning))
    o.stop_at_goal = int(bool(stop_at_goal))
    o.fingerprint = int(bool(fingerprint))
    o.timings = int(bool(timings))
    if max_depth is not None:
        o.max_depth = int(max_depth)
    if max_states is not None:
        o.max_states = int(max_states)
    if expected_states is not None:
        o.expected_states = int(expected_states)
    if stream is not None:
        o.stream = stream
    if comm is not None:
        comm.check()  # a rank that left: fail here, before any launch
        o.comm = comm.handle
        o.world_rank, o.world_size = comm.rank, comm.world
    if max_exchange_records is not None:
        o.max_exchange_records = int(max_exchange_records)
    if shard_from_states is not None:
        o.shard_from_states = int(shard_from_states)
    s = _Search(task, o)
    r = s.run()
    res = BrfsResult(status=STATUS.get(r.status, str(r.status)), states=r.states, expanded=r.expanded,
                     generated=r.generated, num_goal_states=r.num_goal_states, layers=r.layers,
                     layer_counts=[tuple(int(x) for x in row) for row in s.lc], exhausted=bool(r.exhausted),
                     solved=bool(r.solved), goal_id=r.goal_id, fingerprint=r.fingerprint, search_s=r.search_s,
                     words=r.words,
                     stats=DeviceBrfsStats(r.count_ms, r.gen_ms, r.dedup_ms, r.rehashes, 1 << r.table_log2,
                                           r.kernel_launches, r.local_states, r.exchanged, r.exchange_ms,
                                           r.wait_ms),
                     _search=s)
    return res


def hash_rows(states, *, numeric_words: int = 0, stream=None, ctx: Context | None = None):
    """hash::state of each row of a CUDA uint64/int64 tensor [N, W] -> [N] (same dtype). With ``numeric_words`` the
    last numeric_words words of a row are its numeric words, which seed the hash of the (trimmed) atom words."""
    import torch

    from .task import default_context

    if not states.is_cuda or states.dim() != 2 or states.element_size() != 8:
        raise ValueError("hash_rows: states must be a CUDA [N, W] tensor of 64-bit words")
    if numeric_words < 0 or numeric_words > states.shape[1]:
        raise ValueError("hash_rows: numeric_words must be between 0 and the row width")
    states = states.contiguous()
    ctx = ctx or default_context(states.device.index)
    out = torch.empty(states.shape[0], dtype=states.dtype, device=states.device)
    st = stream if stream is not None else torch.cuda.current_stream(states.device).cuda_stream
    check(lib().b2_hash_rows_numeric(ctx.handle, states.data_ptr(), states.shape[0], states.shape[1],
                                     int(numeric_words), out.data_ptr(), st))
    return out


class Heuristic:
    """h^max on the device (mymyr.cuda.Heuristic with kind "max"): grounds the delete relaxation of the task on
    creation; ``evaluate(states)`` returns h of each row (uint32, ``DEAD_END`` for dead ends)."""

    DEAD_END = _lib.B2_DEAD_END

    def __init__(self, task: Task, kind: str = "max"):
        if kind != "max":
            raise ValueError("mymyr_b200 Heuristic: the device evaluates h^max only")
        self.task = task
        h = C.c_void_p()
        check(lib().b2_heuristic_create(task.handle, _lib.B2_HEURISTIC_MAX, C.byref(h)))
        self._h = h
        info = _lib.HeuristicInfo()
        check(lib().b2_heuristic_info_get(h, C.byref(info)))
        self.info = {k: getattr(info, k) for k, _ in _lib.HeuristicInfo._fields_}

    @property
    def handle(self):
        return self._h

    def evaluate(self, states, *, stream=None):
        """h of a CUDA [N, W] tensor of 64-bit words -> [N] int64 (uint32 values; DEAD_END for dead ends)."""
        import torch

        if not states.is_cuda or states.dim() != 2 or states.element_size() != 8:
            raise ValueError("Heuristic.evaluate: states must be a CUDA [N, W] tensor of 64-bit words")
        states = states.contiguous()
        n, W = states.shape
        out = torch.empty(n, dtype=torch.int32, device=states.device)
        st = stream if stream is not None else torch.cuda.current_stream(states.device).cuda_stream
        check(lib().b2_heuristic_evaluate(self._h, states.data_ptr(), W, W, n, out.data_ptr(), st))
        return out.to(torch.int64) & 0xFFFFFFFF

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.b2_heuristic_destroy(h)
        self._h = None


ASTAR_STATUS = {0: "solved", 1: "exhausted", 2: "out_of_states", 3: "unsolvable"}


@dataclass
class AstarResult:
    """search::BestFirstResult's fields for A* (status, cost, plan length, expanded, generated, states, evaluations,
    dead ends, initial h) plus the device's counters."""

    status: str
    cost: float
    plan_length: int
    expanded: int
    generated: int
    states: int
    evaluations: int
    dead_ends: int
    initial_h: float
    waves: int
    f_layers: int
    search_s: float
    stats: dict = field(default_factory=dict)
    _search: object = None
    _owners: tuple = ()  # the task (and shared heuristic) the search reads until it is closed

    @property
    def solved(self) -> bool:
        return self.status == "solved"

    def plan_steps(self):
        """The plan as (parent state, successor index) per step, root first (b2_astar_plan)."""
        n = C.c_uint32()
        check(lib().b2_astar_plan(self._search, None, None, 0, C.byref(n)))
        p = np.zeros(n.value, np.uint32)
        k = np.zeros(n.value, np.uint32)
        check(lib().b2_astar_plan(self._search, p.ctypes.data, k.ctypes.data, n.value, C.byref(n)))
        return p, k

    def plan(self, task: Task):
        """The plan's actions as (schema index, binding) and its states, replayed from the initial state with the
        batched expand (the successor index is a position in canonical order)."""
        import torch

        from . import rl

        _, idx = self.plan_steps()
        row = torch.from_numpy(task.initial_state().view(np.int64)).reshape(1, -1).to(f"cuda:{task.ctx.device}")
        actions, states = [], [row.cpu().numpy().view(np.uint64)[0].copy()]
        for k in idx:
            e = rl.expand(task, row, succ=True)
            j = int(e.offsets[0]) + int(k)
            actions.append((int(e.schema[j]), tuple(int(x) for x in e.binding[j].tolist() if x >= 0)))
            row = e.succ[j: j + 1].clone()
            states.append(row.cpu().numpy().view(np.uint64)[0].copy())
        return actions, states

    def close(self):
        if self._search is not None and _lib._lib is not None:
            _lib._lib.b2_astar_destroy(self._search)
        self._search = None
        self._owners = ()

    def __del__(self):
        self.close()


def astar(task: Task, ctx: Context | None = None, heuristic="max", *, witness_pruning: bool = False,
          max_expansions: int | None = None, expected_states: int | None = None, timings: bool = False,
          stream=None, chunk_candidates: int | None = None, comm=None) -> AstarResult:
    """Eager A* with h^max and unit costs on the device (mymyr.cuda.astar / search::astar_eager): the optimal plan
    cost. ``heuristic`` is "max" or a ``Heuristic`` of the same task (to share its grounding). ``chunk_candidates``
    bounds the successors staged at once (an f layer with more is expanded in chunks; default 2^26). ``comm`` (a
    ``mymyr_b200.dist.Communicator``) partitions the states over its ranks by state-hash owner: every rank calls astar
    together and gets the same result (no plan)."""
    if ctx is not None and task.ctx is not None and ctx.device != task.ctx.device:
        raise ValueError("mymyr_b200 astar: the task lives on another device than ctx")
    o = _lib.AstarOptions()
    lib().b2_astar_options_default(C.byref(o))
    o.witness_pruning = int(bool(witness_pruning))
    o.timings = int(bool(timings))
    if max_expansions is not None:
        o.max_expansions = int(max_expansions)
    if expected_states is not None:
        o.expected_states = int(expected_states)
    if stream is not None:
        o.stream = stream
    if chunk_candidates is not None:
        o.chunk_candidates = int(chunk_candidates)
    if comm is not None:
        comm.check()
        o.comm = comm.handle
    if isinstance(heuristic, Heuristic):
        o.heuristic = heuristic.handle
    elif heuristic != "max":
        raise ValueError("mymyr_b200 astar: the device runs h^max only")
    h = C.c_void_p()
    check(lib().b2_astar_create(task.handle, C.byref(o), C.byref(h)))
    r = _lib.AstarResult()
    try:
        check(lib().b2_astar_run(h, C.byref(r)))
    except Exception:
        lib().b2_astar_destroy(h)
        raise
    stats = {k: getattr(r, k) for k in ("count_ms", "expand_ms", "insert_ms", "eval_ms", "kernel_launches",
                                        "relaxed_ops", "relaxed_atoms")}
    return AstarResult(status=ASTAR_STATUS.get(r.status, str(r.status)), cost=r.cost, plan_length=r.plan_length,
                       expanded=r.expanded, generated=r.generated, states=r.states, evaluations=r.evaluations,
                       dead_ends=r.dead_ends, initial_h=r.initial_h, waves=r.waves, f_layers=r.f_layers,
                       search_s=r.search_s, stats=stats, _search=h, _owners=(task, heuristic, comm))
