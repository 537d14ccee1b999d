"""Test infrastructure: ctypes access to the CPU restatement of the reference's hot path (oracle/port/port.cpp,
built by ``make -C oracle port`` into oracle/_port/libb2_port.so). Imported only by tests/ and smoke()."""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_port" / "libb2_port.so"
_L = None


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _L
    if _L is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"port oracle not built: {LIB_PATH} (run make -C oracle port)")
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.port_last_error.restype = C.c_char_p
        L.port_task_open.restype = P
        L.port_task_open.argtypes = [C.c_char_p]
        L.port_task_close.argtypes = [P]
        L.port_task_info.argtypes = [P, P]
        L.port_initial_state.restype = C.c_int64
        L.port_initial_state.argtypes = [P, P]
        L.port_hash.restype = C.c_uint64
        L.port_hash.argtypes = [P, C.c_uint32]
        L.port_philox_bits64.restype = C.c_uint64
        L.port_philox_bits64.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        L.port_brfs.restype = C.c_int64
        L.port_brfs.argtypes = [P, C.c_uint32, C.c_int, P, P, C.c_uint32, P, C.c_uint64]
        L.port_expand.restype = C.c_int64
        L.port_expand.argtypes = [P, P, C.c_uint64, C.c_int, P, P, P, C.c_uint32, P, C.c_uint64]
        L.port_env_run.restype = C.c_int64
        L.port_env_run.argtypes = [P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint64, P, P]
        _L = L
    return _L


def _check(rc):
    if rc < 0:
        raise RuntimeError("port: " + lib().port_last_error().decode(errors="replace"))
    return rc


class PortTask:
    def __init__(self, text: str):
        self.h = lib().port_task_open(text.encode())
        if not self.h:
            raise RuntimeError("port: " + lib().port_last_error().decode(errors="replace"))
        info = np.zeros(2, np.uint64)
        lib().port_task_info(self.h, info.ctypes.data)
        self.words, self.fluent_slots = int(info[0]), int(info[1])

    def __del__(self):
        if getattr(self, "h", None):
            lib().port_task_close(self.h)
            self.h = None

    def initial_state(self):
        row = np.zeros(self.words, np.uint64)
        _check(lib().port_initial_state(self.h, row.ctypes.data))
        return row

    def brfs(self, max_depth=None, witness_pruning=True, rows=False, row_cap=1 << 20):
        out = np.zeros(6, np.uint64)
        cap = 4096
        lc = np.zeros((cap, 3), np.uint64)
        rbuf = np.zeros((row_cap, self.words), np.uint64) if rows else None
        n = _check(lib().port_brfs(self.h, 0xFFFFFFFF if max_depth is None else max_depth, int(witness_pruning),
                                   out.ctypes.data, lc.ctypes.data, cap, None if rbuf is None else rbuf.ctypes.data,
                                   row_cap if rows else 0))
        r = dict(zip(["states", "expanded", "generated", "num_goal_states", "layers", "fingerprint"],
                     (int(x) for x in out)))
        r["layer_counts"] = [tuple(int(x) for x in row) for row in lc[:n]]
        if rows:
            r["rows"] = rbuf[: r["states"]]
        return r

    def expand(self, states, witness_pruning=False, label_width=8):
        states = np.ascontiguousarray(states, np.uint64)
        n = states.shape[0]
        offsets = np.zeros(n + 1, np.int32)
        m = _check(lib().port_expand(self.h, states.ctypes.data, n, int(witness_pruning), offsets.ctypes.data, None,
                                     None, label_width, None, 0))
        schema = np.zeros(m, np.int32)
        binding = np.zeros((m, label_width), np.int32)
        sh = np.zeros(m, np.uint64)
        _check(lib().port_expand(self.h, states.ctypes.data, n, int(witness_pruning), offsets.ctypes.data,
                                 schema.ctypes.data, binding.ctypes.data, label_width, sh.ctypes.data, m))
        return dict(offsets=offsets, schema=schema, binding=binding, succ_hash=sh, generated=m)

    def env_run(self, rows, steps, seed=0, first_env=0):
        st = np.zeros((rows, self.words), np.uint64)
        rs = np.zeros(rows, np.float32)
        _check(lib().port_env_run(self.h, rows, steps, seed, first_env, st.ctypes.data, rs.ctypes.data))
        return st, rs


def hash_row(row) -> int:
    row = np.ascontiguousarray(row, np.uint64)
    return int(lib().port_hash(row.ctypes.data, len(row)))
