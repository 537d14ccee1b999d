"""Tasks and device contexts of the device path.

``Task.from_text_file(path)`` / ``Task.from_text(text)`` read the reference's normalized task text format
(include/mymyr/formalism/text_format.hpp in maichmueller/mymyr) and compile it with the dense canonical atom layout
(slot = canonical id, TaskOptions::Atoms::Dense). ``Context(device)`` mirrors mymyr.cuda.Context: one per device,
shared by default.
"""

from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _lib
from ._lib import check, lib

_contexts: dict[int, "Context"] = {}
_ctx_lock = threading.Lock()


class Context:
    """A device context (cuda::DeviceContext::create, include/mymyr/cuda/runtime.hpp:148)."""

    def __init__(self, device: int = 0):
        self.device = int(device)
        h = C.c_void_p()
        check(lib().b2_ctx_create(self.device, C.byref(h)))
        self._h = h

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.b2_ctx_destroy(h)
            self._h = None


def default_context(device: int | None = None) -> Context:
    if device is None:
        import torch

        device = torch.cuda.current_device()
    with _ctx_lock:
        c = _contexts.get(device)
        if c is None:
            c = _contexts[device] = Context(device)
        return c


class Task:
    """A compiled task. On a device context (``ctx``) it can run kernels; with ``host_only=True`` it is compiled on
    the host only (layout, initial state, slot records; no GPU needed)."""

    def __init__(self, text: str, ctx: Context | None = None, host_only: bool = False, matcher: str = "auto"):
        L = lib()
        desc = C.POINTER(_lib.TaskDesc)()
        raw = text.encode()
        check(L.b2_task_desc_read_text(raw, len(raw), C.byref(desc)))
        try:
            self.ctx = None if host_only else (ctx or default_context())
            h = C.c_void_p()
            opts = _lib.TaskOptions(_lib.MATCHER[matcher])
            check(L.b2_task_create_ex(self.ctx.handle if self.ctx else None, desc, C.byref(opts), C.byref(h)))
            self._h = h
            self.matcher = "interpreted" if matcher == "interpreted" or host_only else "compiled"
        finally:
            L.b2_task_desc_free(desc)
        info = _lib.TaskInfo()
        check(L.b2_task_info_get(self._h, C.byref(info)))
        self.words = info.words
        self.fluent_slots = info.fluent_slots
        self.num_schemas = info.num_schemas
        self.num_objects = info.num_objects
        self.label_width = info.label_width
        self.object_words = info.object_words
        self.text = text

    @classmethod
    def from_text(cls, text: str, ctx: Context | None = None, host_only: bool = False,
                  matcher: str = "auto") -> "Task":
        return cls(text, ctx, host_only, matcher)

    @classmethod
    def from_text_file(cls, path, ctx: Context | None = None, host_only: bool = False,
                       matcher: str = "auto") -> "Task":
        with open(path) as f:
            return cls(f.read(), ctx, host_only, matcher)

    def compile(self) -> str:
        """Compiles the task's kernels for sm_100a (no device needed) and returns the generated source."""
        n = C.c_size_t()
        check(lib().b2_task_compile(self._h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        check(lib().b2_task_compile(self._h, buf, n.value + 1, None))
        return buf.value.decode()

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def words_(self) -> int:
        return self.words

    def initial_state(self) -> np.ndarray:
        """The initial state row (Task::initial_state), [words] uint64."""
        row = np.zeros(self.words, np.uint64)
        check(lib().b2_task_initial_state(self._h, row.ctypes.data, self.words))
        return row

    def slot_atom(self, slot: int) -> tuple[int, tuple[int, ...]]:
        """(predicate, objects) of fluent slot `slot` (AtomIndex::record)."""
        buf = np.full(66, 0xFFFFFFFF, np.uint32)
        check(lib().b2_task_slot_atom(self._h, slot, buf.ctypes.data, 66))
        args = tuple(int(x) for x in buf[1:] if x != 0xFFFFFFFF)
        return int(buf[0]), args

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.b2_task_destroy(h)
            self._h = None
