"""mymyr_b200: the B200 (sm_100a) device path of the mymyr lifted planner.

Batched lifted successor generation, 64-bit state hashing with device hash-set dedup of BrFS layers, and the batched
RL env step, as hand-written CUDA behind the C ABI of include/mymyr_b200.h. The Python API mirrors the reference's
(mymyr.cuda.brfs, mymyr.rl.expand, mymyr.rl.torch.BatchedEnv, mymyr.hash_rows).
"""

from ._lib import CapacityError, DeviceFault, UnsupportedTask, lib
from .task import Context, Task, default_context

__all__ = ["Task", "Context", "default_context", "lib", "CapacityError", "DeviceFault", "UnsupportedTask"]
__version__ = "0.1.0"
