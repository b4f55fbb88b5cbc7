"""B200-native IQ_K routed-expert hot path (drop-in for mlx-iqk's IqkSwitchLinear).

Hand-written sm_100a CUDA kernels behind a C ABI (``include/iqk_b200.h``,
``libiqk_b200.so``), reached from this thin PyTorch layer. Nothing here falls
back to the CPU: a missing library raises.
"""

from . import format  # noqa: F401
from .format import IqkFormatError
from .kernels import IqkKernelError, IqkRuntimeError
from .nn import DECODE_MAT_LIMIT, IqkSwitchLinear, grid_table, member_table, value_table
from .glu import GraphedSwitchGLU, IqkSwitchGLU

__all__ = ["DECODE_MAT_LIMIT", "IqkFormatError", "IqkKernelError", "IqkRuntimeError",
           "GraphedSwitchGLU", "IqkSwitchGLU", "IqkSwitchLinear", "format", "grid_table", "member_table",
           "value_table"]
