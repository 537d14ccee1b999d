"""RL primitives on the device: ``expand`` (mymyr.rl.expand, python/src/rl_bindings.cpp:2166 in maichmueller/mymyr) and
``BatchedEnv`` (mymyr.rl.torch.BatchedEnv reset/step, python/src/rl_torch_bindings.cpp:827-880), over torch CUDA
tensors. Rows are uint64 words stored in int64 tensors (torch's 64-bit integer type); the bits are the reference's."""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib
from .task import Task


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device, stream):
    return stream if stream is not None else torch.cuda.current_stream(device).cuda_stream


@dataclass
class Expansion:
    """CSR successors of a batch (rl::Expansion, include/mymyr/rl/expand.hpp:92-122)."""

    offsets: torch.Tensor     # [N + 1] int32
    parent: torch.Tensor      # [M] int32
    schema: torch.Tensor      # [M] int32
    binding: torch.Tensor     # [M, label_width] int32 (-1 past the arity)
    succ_hash: torch.Tensor | None  # [M] int64 (uint64 bits of State::hash())
    succ: torch.Tensor | None       # [M, W] int64
    generated: int


def expand(task: Task, states: torch.Tensor, *, canonical_order: bool = True, witness_pruning: bool = False,
           hashes: bool = True, succ: bool = False, capacity: int | None = None, stream=None) -> Expansion:
    """The successors of states [N, W] (CUDA, 64-bit words) in canonical order (also for ``canonical_order=False``,
    which leaves the order to the matcher). ``capacity`` bounds the rows written (None: a count pass sizes the
    outputs exactly)."""
    if not states.is_cuda or states.dim() != 2 or states.element_size() != 8:
        raise ValueError("expand: states must be a CUDA [N, W] tensor of 64-bit words")
    states = states.contiguous()
    n, W = states.shape
    dev = states.device
    st = _stream(dev, stream)
    L = lib()
    offsets = torch.empty(n + 1, dtype=torch.int32, device=dev)
    if capacity is None:
        probe = _lib.Expansion()
        probe.capacity = 0
        probe.offsets = offsets.data_ptr()
        check(L.b2_expand(task.handle, states.data_ptr(), n, W, int(witness_pruning), C.byref(probe), st))
        capacity = probe.generated
    lw = max(1, task.label_width)
    parent = torch.empty(capacity, dtype=torch.int32, device=dev)
    schema = torch.empty(capacity, dtype=torch.int32, device=dev)
    binding = torch.empty((capacity, lw), dtype=torch.int32, device=dev)
    sh = torch.empty(capacity, dtype=torch.int64, device=dev) if hashes else None
    sc = torch.empty((capacity, W), dtype=torch.int64, device=dev) if succ else None
    e = _lib.Expansion()
    e.capacity = capacity
    e.words = W
    e.label_width = lw
    e.succ = _ptr(sc)
    e.parent = parent.data_ptr()
    e.schema = schema.data_ptr()
    e.binding = binding.data_ptr()
    e.offsets = offsets.data_ptr()
    e.succ_hash = _ptr(sh)
    check(L.b2_expand(task.handle, states.data_ptr(), n, W, int(witness_pruning), C.byref(e), st))
    m = e.generated
    return Expansion(offsets, parent[:m], schema[:m], binding[:m], None if sh is None else sh[:m],
                     None if sc is None else sc[:m], m)


class BatchedEnv:
    """Batched environments over one task on a CUDA device (rl::HostEnv semantics, Index action space): every array
    is owned here as a torch tensor and updated in place by reset() and step()."""

    def __init__(self, task: Task, num_envs: int, *, seed: int = 0, max_steps: int = 0, step_reward: float = 0.0,
                 goal_reward: float = 1.0, dead_end_reward: float = 0.0, dead_end: str = "no_successors",
                 dead_end_terminal: bool = True, autoreset: bool = True, witness_pruning: bool = False,
                 first_env: int = 0, device=None):
        self.task = task
        self.device = torch.device(device) if device is not None else torch.device("cuda", task.ctx.device)
        cfg = _lib.EnvConfig()
        lib().b2_env_config_default(C.byref(cfg))
        cfg.seed = seed
        cfg.max_steps = max_steps
        cfg.step_reward = step_reward
        cfg.goal_reward = goal_reward
        cfg.dead_end_reward = dead_end_reward
        cfg.dead_end_none = 1 if dead_end == "none" else 0
        cfg.dead_end_terminal = int(dead_end_terminal)
        cfg.autoreset = int(autoreset)
        cfg.witness_pruning = int(witness_pruning)
        h = C.c_void_p()
        check(lib().b2_env_create(task.handle, C.byref(cfg), C.byref(h)))
        self._h = h
        n, W, d = num_envs, task.words, self.device
        self.num_envs = n
        self.first_env = first_env
        self.states = torch.zeros((n, W), dtype=torch.int64, device=d)
        self.steps = torch.zeros(n, dtype=torch.int32, device=d)
        self.draws = torch.zeros(n, dtype=torch.int64, device=d)
        self.at_goal = torch.zeros(n, dtype=torch.uint8, device=d)
        self.counts = torch.zeros((n, max(1, task.num_schemas)), dtype=torch.int32, device=d)
        lw = max(1, task.label_width)
        self.reward = torch.zeros(n, dtype=torch.float32, device=d)
        self.terminated = torch.zeros(n, dtype=torch.uint8, device=d)
        self.truncated = torch.zeros(n, dtype=torch.uint8, device=d)
        self.count = torch.zeros(n, dtype=torch.int32, device=d)
        self.final_states = torch.zeros((n, W), dtype=torch.int64, device=d)
        self.schema = torch.zeros(n, dtype=torch.int32, device=d)
        self.binding = torch.zeros((n, lw), dtype=torch.int32, device=d)
        self.invalid = torch.zeros(n, dtype=torch.uint8, device=d)
        self.goal = torch.zeros(n, dtype=torch.uint8, device=d)
        self._batch = _lib.EnvBatch(self.states.data_ptr(), n, W, self.steps.data_ptr(), self.draws.data_ptr(),
                                    self.at_goal.data_ptr(), self.counts.data_ptr(), first_env)
        self._out = _lib.StepOut(self.reward.data_ptr(), self.terminated.data_ptr(), self.truncated.data_ptr(),
                                 self.count.data_ptr(), self.final_states.data_ptr(), self.schema.data_ptr(),
                                 self.binding.data_ptr(), lw, self.invalid.data_ptr(), self.goal.data_ptr())

    def reset(self, mask: torch.Tensor | None = None, stream=None):
        """Resets the rows with mask[i] (all rows without a mask) to the initial state; draw counters are kept."""
        check(lib().b2_env_reset(self._h, C.byref(self._batch), _ptr(mask), self.count.data_ptr(),
                                 _stream(self.device, stream)))
        return self.states

    def step(self, action: torch.Tensor | None = None, stream=None, next_task_ids: torch.Tensor | None = None):
        """One step of every environment: action [N] int64 indexes the canonical successor order (None: the random
        policy). Outputs land in this object's tensors (reward, terminated, truncated, count, final_states, schema,
        binding, invalid, goal). ``next_task_ids`` [N] int32 (device) names the task an autoresetting row restarts
        in; the env has one task (id 0), and another id is reported by check_errors() (ValueError) while the row
        keeps its task."""
        if action is not None and (action.dtype != torch.int64 or not action.is_cuda):
            raise ValueError("step: action must be a CUDA int64 tensor")
        if next_task_ids is not None and (next_task_ids.dtype != torch.int32 or not next_task_ids.is_cuda or
                                          next_task_ids.numel() != self.num_envs):
            raise ValueError("step: next_task_ids must be a CUDA int32 tensor of num_envs entries")
        check(lib().b2_env_step_ex(self._h, C.byref(self._batch), C.byref(self._out), _ptr(action),
                                   _ptr(next_task_ids), _stream(self.device, stream)))
        return self.states

    def check_errors(self):
        """Synchronizes the device and raises what the steps since the last check flagged: RuntimeError for a state
        whose count cache did not match it (states written without reset()), ValueError for next_task_ids outside
        the env's tasks (cuda::DeviceEnv::check_errors)."""
        check(lib().b2_env_check_errors(self._h))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.b2_env_destroy(h)
            self._h = None
