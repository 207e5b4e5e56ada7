"""lancius_b200 -- B200 (sm_100a) execution backend for the Lancius static-graph IR.

The IR, wave scheduler and memory planner are C11 (csrc/host), the kernels and
the executor are CUDA for sm_100a (csrc/cuda); both are linked into the in-tree
liblancius_b200.so, whose C ABI is include/lancius_cuda.h. This Python layer
only binds that library.
"""
from ._lib import LIB_PATH, load  # noqa: F401
from .graph import Graph, LanciusError, Node, Schedule  # noqa: F401
from .runtime import EPI_GELU, EPI_NONE, EPI_RELU, MODE_FP32_EXACT, MODE_TF32, MODE_BF16, Device  # noqa: F401
