"""fastmd_b200: FastMD's per-step MD hot path on hand-written sm_100a kernels (libfastmd_b200.so).

Surfaces mirroring the reference: ``ops`` (fastmd.ops), ``graph`` (fastmd.graph builders),
``energy_derivative`` (fastmd.engine), ``gpu_nhc`` and ``whole_step`` (fastmd.execution /
fastmd.interfaces), ``mace`` (the MACE-architecture energy tap).
"""
from fastmd_b200 import (  # noqa: F401
    _lib, decomposed_indexed_cat_silu_linear, energy_derivative, gpu_nhc, graph, mace, ops, segment_attention, units,
    whole_step, wide_gemm)

__all__ = ["decomposed_indexed_cat_silu_linear", "energy_derivative", "gpu_nhc", "graph", "mace", "ops",
           "segment_attention", "units", "whole_step", "wide_gemm"]
