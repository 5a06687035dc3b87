"""opennpu_b200: OpenNPU's int4 group-32 weight-only matmul path, rebuilt for NVIDIA B200.

The compute is libonpu.so (CUDA for sm_100a, built in-tree by ``python -m opennpu_b200.build``),
reached through the reference's onpu_* C ABI (``libonpu``), the reference engine's Python call
shapes (``npu4``) or torch device tensors (``dense``). There is no CPU fallback: importing the
device paths without the built library, or running them without a B200, raises.
"""
from .libonpu import OnpuError, load, last_error  # noqa: F401

__all__ = ["OnpuError", "load", "last_error"]
