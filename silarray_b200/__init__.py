"""silarray_b200: a B200 (sm_100a) backend for silarray's sil:: array ops.

    include/silcu.h        the C ABI (the drop-in boundary for include/gpu.h)
    silarray_b200/csrc/    the CUDA kernels behind it
    silarray_b200.gpu      Python mirror of silarray's `class gpu`
    silarray_b200.transformer, .dist   composed workloads and the multi-GPU partitioner
"""
from ._lib import SilcuError, lib  # noqa: F401

__all__ = ["SilcuError", "lib"]
