"""Test infrastructure: ctypes access to the reference planner's CPU path (oracle/_ref/libref_oracle.so, built from the
reference's sources by oracle/Makefile; see ref_oracle.cpp for the reference call behind each function).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module. It is the checker, never the
product: nothing in mymyr_b200/ imports it.
"""

from __future__ import annotations

import ctypes as C
import os
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "libref_oracle.so"

_L = None


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _L
    if _L is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"reference oracle not built: {LIB_PATH} (run make -C oracle)")
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.ref_last_error.restype = C.c_char_p
        L.ref_task_open.restype = P
        L.ref_task_open.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_task_close.argtypes = [P]
        for name in ("ref_task_info", "ref_initial_state", "ref_is_goal", "ref_brfs", "ref_brfs_states", "ref_expand",
                     "ref_env_reset", "ref_env_step", "ref_pool_bench", "ref_astar", "ref_hmax", "ref_ground_stats", "ref_brfs_limited"):
            getattr(L, name).restype = C.c_int64
        L.ref_task_info.argtypes = [P, P]
        L.ref_initial_state.argtypes = [P, P, C.c_uint32]
        L.ref_hash_state.restype = C.c_uint64
        L.ref_hash_state.argtypes = [P, C.c_uint32]
        L.ref_hash_state_numeric.restype = C.c_uint64
        L.ref_hash_state_numeric.argtypes = [P, C.c_uint32, C.c_uint32]
        L.ref_canonical_hash.restype = C.c_uint64
        L.ref_canonical_hash.argtypes = [P, P, C.c_uint32]
        L.ref_philox_bits64.restype = C.c_uint64
        L.ref_philox_bits64.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32]
        L.ref_philox_block.argtypes = [C.c_uint32] * 6 + [P]
        L.ref_brfs.argtypes = [P, C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_int, P, P, P, C.c_uint32, C.c_int]
        L.ref_brfs_states.argtypes = [P, C.c_uint32, C.c_int, P, C.c_uint64, C.c_uint32, P, P]
        L.ref_expand.argtypes = [P, P, C.c_uint64, C.c_uint32, C.c_int, C.c_int, C.c_uint32, P, P, P, P, C.c_uint32, P,
                                 P, C.c_uint64, P]
        L.ref_env_create.restype = P
        L.ref_env_create.argtypes = [P, C.c_uint64, C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_int, C.c_int,
                                     C.c_int, C.c_uint32]
        L.ref_env_destroy.argtypes = [P]
        L.ref_env_reset.argtypes = [P, P, C.c_uint64, C.c_uint32, P, P, P, P]
        L.ref_env_step.argtypes = [P, P, C.c_uint64, C.c_uint32, P, P, P, C.c_uint64, P, P, P, P, P, P, P, P,
                                   C.c_uint32, P, P, P]
        L.ref_pool_bench.argtypes = [P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, P, P]
        L.ref_astar.argtypes = [P, P, P]
        L.ref_hmax.argtypes = [P, P, C.c_uint64, C.c_uint32, P]
        L.ref_ground_stats.argtypes = [P, P]
        L.ref_brfs_limited.argtypes = [P, C.c_uint64, C.c_uint32, C.c_int, C.c_int, C.c_int, P, P, C.c_uint32]
        _L = L
    return _L


def _check(rc):
    if rc < 0:
        raise RuntimeError("reference: " + lib().ref_last_error().decode(errors="replace"))
    return rc


def _p(a):
    return None if a is None else a.ctypes.data


class RefTask:
    """A reference Task (Task::from_text_file) with dense atom slots by default (the device path's layout)."""

    def __init__(self, text: str, atoms: str = "dense"):
        mode = {"auto": 0, "reachable": 1, "dense": 2}[atoms]
        fd, path = tempfile.mkstemp(suffix=".txt")
        try:
            with os.fdopen(fd, "w") as f:
                f.write(text)
            self.h = lib().ref_task_open(path.encode(), mode, 0)
        finally:
            os.unlink(path)
        if not self.h:
            raise RuntimeError("reference: " + lib().ref_last_error().decode(errors="replace"))
        info = np.zeros(8, np.uint64)
        _check(lib().ref_task_info(self.h, info.ctypes.data))
        self.words, self.fluent_slots, self.num_schemas, self.num_objects = (int(x) for x in info[:4])
        self.label_width = int(info[7])

    def __del__(self):
        if getattr(self, "h", None):
            lib().ref_task_close(self.h)
            self.h = None

    def initial_state(self) -> np.ndarray:
        row = np.zeros(self.words, np.uint64)
        _check(lib().ref_initial_state(self.h, row.ctypes.data, self.words))
        return row

    def is_goal(self, row: np.ndarray) -> bool:
        row = np.ascontiguousarray(row, np.uint64)
        return bool(_check(lib().ref_is_goal(self.h, row.ctypes.data, len(row))))

    def canonical_hash(self, row: np.ndarray) -> int:
        row = np.ascontiguousarray(row, np.uint64)
        return int(lib().ref_canonical_hash(self.h, row.ctypes.data, len(row)))

    def brfs(self, threads=1, max_depth=None, stop_at_goal=True, witness_pruning=True, fingerprint=False,
             store="auto"):
        out = np.zeros(10, np.uint64)
        sec = C.c_double()
        cap = 4096
        lc = np.zeros((cap, 3), np.uint64)
        n = _check(lib().ref_brfs(self.h, threads, 0xFFFFFFFF if max_depth is None else max_depth, int(stop_at_goal),
                                  int(witness_pruning), int(fingerprint), out.ctypes.data, C.byref(sec),
                                  lc.ctypes.data, cap, {"auto": 0, "flat": 1, "concurrent": 4}[store]))
        keys = ["states", "expanded", "generated", "num_goal_states", "layers", "exhausted", "solved", "fingerprint",
                "plan_length", "status"]
        r = {k: int(v) for k, v in zip(keys, out)}
        r["layer_counts"] = [tuple(int(x) for x in row) for row in lc[:n]]
        r["search_s"] = sec.value
        return r

    def brfs_limited(self, max_states, max_depth=None, stop_at_goal=True, witness_pruning=True, fingerprint=False):
        """Single-threaded mymyr::brfs with max_states (status as SearchStatus: 0 solved, 1 exhausted, 2 out of
        states, 6 unsolvable)."""
        out = np.zeros(10, np.uint64)
        cap = 4096
        lc = np.zeros((cap, 3), np.uint64)
        n = _check(lib().ref_brfs_limited(self.h, max_states, 0xFFFFFFFF if max_depth is None else max_depth,
                                          int(stop_at_goal), int(witness_pruning), int(fingerprint), out.ctypes.data,
                                          lc.ctypes.data, cap))
        keys = ["states", "expanded", "generated", "num_goal_states", "layers", "exhausted", "solved", "fingerprint",
                "plan_length", "status"]
        r = {k: int(v) for k, v in zip(keys, out)}
        r["layer_counts"] = [tuple(int(x) for x in row) for row in lc[:n]]
        return r

    def brfs_states(self, max_depth=None, witness_pruning=True, cap=1 << 22):
        rows = np.zeros((cap, self.words), np.uint64)
        par = np.zeros(cap, np.uint32)
        idx = np.zeros(cap, np.uint32)
        n = _check(lib().ref_brfs_states(self.h, 0xFFFFFFFF if max_depth is None else max_depth, int(witness_pruning),
                                         rows.ctypes.data, cap, self.words, par.ctypes.data, idx.ctypes.data))
        if n == -2:
            raise RuntimeError("ref_brfs_states: capacity")
        return rows[:n], par[:n], idx[:n]

    def expand(self, states: np.ndarray, witness_pruning=False, canonical=True, threads=1, succ=False,
               capacity=None):
        states = np.ascontiguousarray(states, np.uint64)
        n, W = states.shape
        offsets = np.zeros(n + 1, np.int32)
        sec = C.c_double()
        if capacity is None:
            capacity = _check(lib().ref_expand(self.h, states.ctypes.data, n, W, int(witness_pruning), int(canonical),
                                               threads, offsets.ctypes.data, None, None, None, 1, None, None, 0,
                                               C.byref(sec)))
        lw = max(1, self.label_width)
        parent = np.zeros(capacity, np.int32)
        schema = np.zeros(capacity, np.int32)
        binding = np.zeros((capacity, lw), np.int32)
        sh = np.zeros(capacity, np.uint64)
        sc = np.zeros((capacity, W), np.uint64) if succ else None
        m = _check(lib().ref_expand(self.h, states.ctypes.data, n, W, int(witness_pruning), int(canonical), threads,
                                    offsets.ctypes.data, parent.ctypes.data, schema.ctypes.data, binding.ctypes.data,
                                    lw, sh.ctypes.data, _p(sc), capacity, C.byref(sec)))
        return dict(offsets=offsets, parent=parent[:m], schema=schema[:m], binding=binding[:m], succ_hash=sh[:m],
                    succ=None if sc is None else sc[:m], generated=m, seconds=sec.value)

    def astar(self):
        out = np.zeros(5, np.float64)
        sec = C.c_double()
        _check(lib().ref_astar(self.h, out.ctypes.data, C.byref(sec)))
        return dict(solved=bool(out[0]), cost=out[1], plan_length=int(out[2]), expanded=int(out[3]),
                    generated=int(out[4]), seconds=sec.value)

    def hmax(self, rows: np.ndarray) -> np.ndarray:
        """h^max (unit costs, grounded) of each row; +inf for dead ends."""
        rows = np.ascontiguousarray(rows, np.uint64)
        out = np.zeros(rows.shape[0], np.float64)
        _check(lib().ref_hmax(self.h, rows.ctypes.data, rows.shape[0], rows.shape[1], out.ctypes.data))
        return out

    def ground_stats(self) -> dict:
        out = np.zeros(5, np.uint64)
        _check(lib().ref_ground_stats(self.h, out.ctypes.data))
        return dict(zip(["reached_atoms", "ground_actions", "operators", "propositions", "rounds"],
                        (int(x) for x in out)))

    def pool_bench(self, num_envs, steps, threads, seed=0):
        sec = C.c_double()
        h = C.c_uint64()
        _check(lib().ref_pool_bench(self.h, num_envs, steps, threads, seed, C.byref(sec), C.byref(h)))
        return sec.value, h.value


class RefEnv:
    """rl::HostEnv over a RefTask (single instance, Index actions)."""

    def __init__(self, task: RefTask, rows: int, seed=0, max_steps=0, step_reward=0.0, goal_reward=1.0,
                 dead_end_reward=0.0, dead_end_none=False, dead_end_terminal=True, autoreset=True, threads=1,
                 first_env=0):
        self.task = task
        self.h = lib().ref_env_create(task.h, seed, max_steps, step_reward, goal_reward, dead_end_reward,
                                      int(dead_end_none), int(dead_end_terminal), int(autoreset), threads)
        if not self.h:
            raise RuntimeError("reference: " + lib().ref_last_error().decode(errors="replace"))
        W = task.words
        self.rows, self.W, self.first_env = rows, W, first_env
        self.states = np.zeros((rows, W), np.uint64)
        self.steps = np.zeros(rows, np.int32)
        self.draws = np.zeros(rows, np.uint64)
        self.at_goal = np.zeros(rows, np.uint8)
        self.count = np.zeros(rows, np.int32)
        lw = max(1, task.label_width)
        self.lw = lw
        self.reward = np.zeros(rows, np.float32)
        self.terminated = np.zeros(rows, np.uint8)
        self.truncated = np.zeros(rows, np.uint8)
        self.final_states = np.zeros((rows, W), np.uint64)
        self.schema = np.zeros(rows, np.int32)
        self.binding = np.zeros((rows, lw), np.int32)
        self.invalid = np.zeros(rows, np.uint8)
        self.goal = np.zeros(rows, np.uint8)

    def __del__(self):
        if getattr(self, "h", None):
            lib().ref_env_destroy(self.h)
            self.h = None

    def reset(self):
        _check(lib().ref_env_reset(self.h, self.states.ctypes.data, self.rows, self.W, self.steps.ctypes.data,
                                   self.draws.ctypes.data, self.at_goal.ctypes.data, self.count.ctypes.data))

    def step(self, actions: np.ndarray | None = None) -> float:
        sec = C.c_double()
        a = None if actions is None else np.ascontiguousarray(actions, np.int64)
        _check(lib().ref_env_step(self.h, self.states.ctypes.data, self.rows, self.W, self.steps.ctypes.data,
                                  self.draws.ctypes.data, self.at_goal.ctypes.data, self.first_env, _p(a),
                                  self.reward.ctypes.data, self.terminated.ctypes.data, self.truncated.ctypes.data,
                                  self.count.ctypes.data, self.final_states.ctypes.data, self.schema.ctypes.data,
                                  self.binding.ctypes.data, self.lw, self.invalid.ctypes.data, self.goal.ctypes.data,
                                  C.byref(sec)))
        return sec.value


def hash_state(row: np.ndarray, numeric_words: int = 0) -> int:
    row = np.ascontiguousarray(row, np.uint64)
    if numeric_words:
        return int(lib().ref_hash_state_numeric(row.ctypes.data, len(row), numeric_words))
    return int(lib().ref_hash_state(row.ctypes.data, len(row)))


def philox_bits64(seed, env, draw, purpose=0) -> int:
    return int(lib().ref_philox_bits64(seed, env, draw, purpose))


# ------------------------------------------------------------------------------------------------ reference-side shim
_shim = None


def shim_available() -> bool:
    return (HERE / "_ref" / "libshim_check.so").exists()


def _shim_lib():
    """oracle/_ref/libshim_check.so: include/mymyr_b200_shim.hpp compiled against the reference (oracle/shim_check.cpp)."""
    global _shim
    if _shim is None:
        import mymyr_b200  # the device library first: the shim links it

        mymyr_b200.lib()
        L = C.CDLL(str(HERE / "_ref" / "libshim_check.so"))
        L.shim_check_layout.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
        L.shim_check_layout.restype = C.c_int
        L.shim_check_brfs.argtypes = [C.c_char_p, C.c_int, C.c_uint32, C.c_int, C.c_int, C.c_void_p, C.c_char_p,
                                      C.c_size_t]
        L.shim_check_brfs.restype = C.c_int
        _shim = L
    return _shim


ATOMS = {"auto": 0, "reachable": 1, "dense": 2}


def shim_layout(text: str, atoms: str = "auto") -> tuple[int, str]:
    """The shim's describe() + b2_task_create (host only) against the reference Task's dense twin: (0, "") when
    words, slots and the initial row agree."""
    msg = C.create_string_buffer(1024)
    rc = _shim_lib().shim_check_layout(text.encode(), ATOMS[atoms], msg, 1024)
    return rc, msg.value.decode(errors="replace")


def shim_brfs(text: str, atoms: str = "auto", max_depth=None, witness_pruning=True, stop_at_goal=False):
    """b2shim::brfs (the device) and mymyr::brfs on the same reference Task: (rc, device fields, reference fields,
    message); rc 0 when every field and the per-layer counts agree."""
    out = np.zeros(16, np.uint64)
    msg = C.create_string_buffer(1024)
    rc = _shim_lib().shim_check_brfs(text.encode(), ATOMS[atoms], 0xFFFFFFFF if max_depth is None else max_depth,
                                     int(witness_pruning), int(stop_at_goal), out.ctypes.data, msg, 1024)
    keys = ["states", "expanded", "generated", "num_goal_states", "layers", "fingerprint", "solved", "status"]
    return rc, dict(zip(keys, map(int, out[:8]))), dict(zip(keys, map(int, out[8:]))), msg.value.decode(errors="replace")
