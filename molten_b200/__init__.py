"""molten_b200: a B200-native (sm_100a) backend for Molten's fused-kernel path.

The front end (``ir``, ``fusion``, ``compiler``) keeps the reference's API;
``codegen`` emits hand-structured sm_100a CUDA; ``runtime`` builds cubins
with nvcc and launches them through the C-ABI library ``libmolten_rt.so``.
"""

__version__ = "0.1.0"

from .ir import DataflowGraph, Op, OpType, TensorShape
from .fusion import FusionEngine, FusionGroup
from .codegen import CodeGenerator, GeneratedKernel, KernelConfig, compile_graph
from .compiler import ZeroCompiler

__all__ = [
    "DataflowGraph", "Op", "OpType", "TensorShape",
    "FusionEngine", "FusionGroup",
    "CodeGenerator", "GeneratedKernel", "KernelConfig", "compile_graph",
    "ZeroCompiler",
]
