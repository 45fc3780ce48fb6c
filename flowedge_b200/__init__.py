"""flowedge_b200: B200-native (sm_100a) policy-sampling hot path of FlowEdge.

The product is the C-ABI library `libflowedge_b200.so` (include/flowedge_b200.h),
a drop-in for the reference's `fe_engine_*` entry points.  `engine.Engine` is
its Python binding; `checkpoint` writes synthetic checkpoints in the
reference's converted safetensors layout.
"""

from .engine import Engine, FlowEdgeError, load_library  # noqa: F401

__all__ = ["Engine", "FlowEdgeError", "load_library"]
