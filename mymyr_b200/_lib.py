"""ctypes binding of the C ABI in include/mymyr_b200.h (libmymyr_b200.so, built in-tree by mymyr_b200.build).

There is no fallback: if the library is missing, importing the device API raises. Status codes become the Python
exceptions the reference's nanobind module raises for the same C++ exceptions (std::invalid_argument -> ValueError,
std::length_error -> ValueError, std::runtime_error / CudaError -> RuntimeError).
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmymyr_b200.so"

B2_OK = 0
B2_INVALID_ARGUMENT = 1
B2_UNSUPPORTED = 2
B2_CAPACITY = 3
B2_CUDA_ERROR = 4
B2_DEVICE_FAULT = 5
B2_PARSE_ERROR = 6


class DeviceFault(RuntimeError):
    """A kernel reported a sticky status bit (a probe bound or a bounded wait ran out)."""


class CapacityError(ValueError):
    """An output or arena capacity is too small (std::length_error in the reference)."""


class UnsupportedTask(ValueError):
    """The task has features the device path does not run."""


class Literal(C.Structure):
    _fields_ = [("pred", C.c_uint32), ("positive", C.c_uint32), ("term_begin", C.c_uint32), ("term_count", C.c_uint32)]


class SchemaDesc(C.Structure):
    _fields_ = [("arity", C.c_uint32), ("pre_begin", C.c_uint32), ("pre_count", C.c_uint32),
                ("eff_begin", C.c_uint32), ("eff_count", C.c_uint32), ("name", C.c_char_p)]


class TaskDesc(C.Structure):
    _fields_ = [("num_objects", C.c_uint32), ("num_predicates", C.c_uint32),
                ("pred_kind", C.POINTER(C.c_uint8)), ("pred_arity", C.POINTER(C.c_uint32)),
                ("terms", C.POINTER(C.c_int32)), ("num_terms", C.c_uint32),
                ("literals", C.POINTER(Literal)), ("num_literals", C.c_uint32),
                ("schemas", C.POINTER(SchemaDesc)), ("num_schemas", C.c_uint32),
                ("static_init", C.POINTER(C.c_uint32)), ("static_init_words", C.c_uint64),
                ("fluent_init", C.POINTER(C.c_uint32)), ("fluent_init_words", C.c_uint64),
                ("goal_begin", C.c_uint32), ("goal_count", C.c_uint32), ("unsupported", C.c_uint32)]


class TaskOptions(C.Structure):
    _fields_ = [("matcher", C.c_int32)]


MATCHER = {"auto": 0, "interpreted": 1, "compiled": 2}


class TaskInfo(C.Structure):
    _fields_ = [("words", C.c_uint32), ("fluent_slots", C.c_uint32), ("num_schemas", C.c_uint32),
                ("num_objects", C.c_uint32), ("label_width", C.c_uint32), ("object_words", C.c_uint32)]


class Expansion(C.Structure):
    _fields_ = [("capacity", C.c_uint64), ("words", C.c_uint32), ("label_width", C.c_uint32),
                ("succ", C.c_void_p), ("parent", C.c_void_p), ("schema", C.c_void_p), ("binding", C.c_void_p),
                ("offsets", C.c_void_p), ("succ_hash", C.c_void_p), ("generated", C.c_uint64)]


class BrfsOptions(C.Structure):
    _fields_ = [("witness_pruning", C.c_int32), ("stop_at_goal", C.c_int32), ("fingerprint", C.c_int32),
                ("max_depth", C.c_uint32), ("max_states", C.c_uint64), ("expected_states", C.c_uint64),
                ("timings", C.c_int32), ("world_rank", C.c_int32), ("world_size", C.c_int32),
                ("stream", C.c_void_p), ("comm", C.c_void_p), ("max_exchange_records", C.c_uint64),
                ("shard_from_states", C.c_uint64)]


class BrfsResult(C.Structure):
    _fields_ = [("status", C.c_uint32), ("layers", C.c_uint32), ("states", C.c_uint64), ("expanded", C.c_uint64),
                ("generated", C.c_uint64), ("num_goal_states", C.c_uint64), ("exhausted", C.c_int32),
                ("solved", C.c_int32), ("goal_id", C.c_uint64), ("fingerprint", C.c_uint64),
                ("search_s", C.c_double), ("count_ms", C.c_double), ("gen_ms", C.c_double),
                ("dedup_ms", C.c_double), ("kernel_launches", C.c_uint64),
                ("layer_counts", C.POINTER(C.c_uint64)), ("layer_capacity", C.c_uint32),
                ("table_log2", C.c_uint32), ("rehashes", C.c_uint32), ("words", C.c_uint32),
                ("local_states", C.c_uint64), ("exchanged", C.c_uint64), ("exchange_ms", C.c_double),
                ("wait_ms", C.c_double)]


class HeuristicInfo(C.Structure):
    _fields_ = [("props", C.c_uint32), ("ops", C.c_uint32), ("reached_atoms", C.c_uint64),
                ("ground_actions", C.c_uint64), ("goal_atoms", C.c_uint32), ("goal_unreachable", C.c_uint32)]


class AstarOptions(C.Structure):
    _fields_ = [("max_expansions", C.c_uint64), ("expected_states", C.c_uint64), ("witness_pruning", C.c_int32),
                ("timings", C.c_int32), ("stream", C.c_void_p), ("heuristic", C.c_void_p),
                ("chunk_candidates", C.c_uint64), ("comm", C.c_void_p)]


class AstarResult(C.Structure):
    _fields_ = [("status", C.c_uint32), ("waves", C.c_uint32), ("cost", C.c_double), ("expanded", C.c_uint64),
                ("generated", C.c_uint64), ("states", C.c_uint64), ("evaluations", C.c_uint64),
                ("dead_ends", C.c_uint64), ("initial_h", C.c_double), ("f_layers", C.c_uint32),
                ("plan_length", C.c_uint32), ("search_s", C.c_double), ("count_ms", C.c_double),
                ("expand_ms", C.c_double), ("insert_ms", C.c_double), ("eval_ms", C.c_double),
                ("kernel_launches", C.c_uint64), ("relaxed_ops", C.c_uint64), ("relaxed_atoms", C.c_uint64)]


B2_HEURISTIC_MAX = 2
B2_DEAD_END = 0xFFFFFFFF


class CommId(C.Structure):
    _fields_ = [("bytes", C.c_char * 128)]


class EnvConfig(C.Structure):
    _fields_ = [("seed", C.c_uint64), ("max_steps", C.c_uint32), ("step_reward", C.c_float),
                ("goal_reward", C.c_float), ("dead_end_reward", C.c_float), ("dead_end_none", C.c_int32),
                ("dead_end_terminal", C.c_int32), ("autoreset", C.c_int32), ("witness_pruning", C.c_int32)]


class EnvBatch(C.Structure):
    _fields_ = [("states", C.c_void_p), ("rows", C.c_uint64), ("words", C.c_uint32), ("steps", C.c_void_p),
                ("draws", C.c_void_p), ("at_goal", C.c_void_p), ("counts", C.c_void_p), ("first_env", C.c_uint64)]


class StepOut(C.Structure):
    _fields_ = [("reward", C.c_void_p), ("terminated", C.c_void_p), ("truncated", C.c_void_p),
                ("count", C.c_void_p), ("final_states", C.c_void_p), ("schema", C.c_void_p),
                ("binding", C.c_void_p), ("label_width", C.c_uint32), ("invalid", C.c_void_p), ("goal", C.c_void_p)]


P = C.c_void_p
PP = C.POINTER(C.c_void_p)
U32, U64, I32 = C.c_uint32, C.c_uint64, C.c_int32

# name -> (restype, argtypes): every entry point declared in include/mymyr_b200.h
SIGNATURES = {
    "b2_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
    "b2_version": (C.c_char_p, []),
    "b2_ctx_create": (C.c_int, [C.c_int, PP]),
    "b2_ctx_destroy": (None, [P]),
    "b2_task_desc_read_text": (C.c_int, [C.c_char_p, C.c_size_t, C.POINTER(C.POINTER(TaskDesc))]),
    "b2_task_desc_free": (None, [C.POINTER(TaskDesc)]),
    "b2_task_create": (C.c_int, [P, C.POINTER(TaskDesc), PP]),
    "b2_task_destroy": (None, [P]),
    "b2_task_create_ex": (C.c_int, [P, C.POINTER(TaskDesc), C.POINTER(TaskOptions), PP]),
    "b2_task_compile": (C.c_int, [P, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "b2_task_info_get": (C.c_int, [P, C.POINTER(TaskInfo)]),
    "b2_task_initial_state": (C.c_int, [P, P, U32]),
    "b2_task_slot_atom": (C.c_int, [P, U32, P, U32]),
    "b2_hash_rows": (C.c_int, [P, P, U64, U32, P, P]),
    "b2_hash_rows_numeric": (C.c_int, [P, P, U64, U32, U32, P, P]),
    "b2_expand": (C.c_int, [P, P, U64, U32, C.c_int, C.POINTER(Expansion), P]),
    "b2_expand_noalloc": (C.c_int, [P, P, U64, U32, C.c_int, C.POINTER(Expansion), P]),
    "b2_comm_id_new": (C.c_int, [C.POINTER(CommId)]),
    "b2_comm_create": (C.c_int, [P, C.POINTER(CommId), U32, U32, PP]),
    "b2_comm_set_timeout": (C.c_int, [P, C.c_double]),
    "b2_comm_destroy": (None, [P]),
    "b2_brfs_options_default": (None, [C.POINTER(BrfsOptions)]),
    "b2_brfs_create": (C.c_int, [P, C.POINTER(BrfsOptions), PP]),
    "b2_brfs_run": (C.c_int, [P, C.POINTER(BrfsResult)]),
    "b2_brfs_states": (C.c_int, [P, U64, U64, P, U32]),
    "b2_brfs_nodes": (C.c_int, [P, U64, U64, P, P]),
    "b2_brfs_state_hashes": (C.c_int, [P, U64, U64, P]),
    "b2_brfs_local_count": (C.c_int, [P, C.POINTER(C.c_uint64)]),
    "b2_brfs_local": (C.c_int, [P, U64, U64, P, P, U32, P, P, P]),
    "b2_brfs_destroy": (None, [P]),
    "b2_heuristic_create": (C.c_int, [P, C.c_int32, PP]),
    "b2_heuristic_info_get": (C.c_int, [P, C.POINTER(HeuristicInfo)]),
    "b2_heuristic_evaluate": (C.c_int, [P, P, U64, U32, U64, P, P]),
    "b2_heuristic_destroy": (None, [P]),
    "b2_astar_options_default": (None, [C.POINTER(AstarOptions)]),
    "b2_astar_create": (C.c_int, [P, C.POINTER(AstarOptions), PP]),
    "b2_astar_run": (C.c_int, [P, C.POINTER(AstarResult)]),
    "b2_astar_plan": (C.c_int, [P, P, P, U32, C.POINTER(C.c_uint32)]),
    "b2_astar_destroy": (None, [P]),
    "b2_env_config_default": (None, [C.POINTER(EnvConfig)]),
    "b2_env_create": (C.c_int, [P, C.POINTER(EnvConfig), PP]),
    "b2_env_reset": (C.c_int, [P, C.POINTER(EnvBatch), P, P, P]),
    "b2_env_step": (C.c_int, [P, C.POINTER(EnvBatch), C.POINTER(StepOut), P, P]),
    "b2_env_step_ex": (C.c_int, [P, C.POINTER(EnvBatch), C.POINTER(StepOut), P, P, P]),
    "b2_env_check_errors": (C.c_int, [P]),
    "b2_env_destroy": (None, [P]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"mymyr_b200: {LIB_PATH} is missing; build it with __graft_entry__.build() "
                               "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(4096)
    lib().b2_last_error(buf, 4096)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status == B2_OK:
        return
    msg = last_error()
    if status == B2_UNSUPPORTED:
        raise UnsupportedTask(msg)
    if status == B2_CAPACITY:
        raise CapacityError(msg)
    if status == B2_INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == B2_DEVICE_FAULT:
        raise DeviceFault(msg)
    raise RuntimeError(msg)
