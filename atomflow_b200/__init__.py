"""AtomFlow-B200: the W8A16 decode hot path (GEMV + lm_head + argmax) for sm_100a.

The product is the CUDA library libatomflow_b200.so behind the C ABI in
include/atomflow_b200.h and the reference-compatible View launchers in
include/atomflow_view_ops.h.  `atomflow_b200.ops` wraps the C ABI for torch
tensors; `atomflow_b200.build` compiles the library in-tree.
"""
from ._lib import (ArgmaxMode, AtomflowError, ScaleKind, Status, WeightDtype, lib, lib_path)

__all__ = ["ArgmaxMode", "AtomflowError", "ScaleKind", "Status", "WeightDtype", "lib", "lib_path"]
