"""fastmd_b200: FastMD's per-step MD hot path on hand-written sm_100a kernels (libfastmd_b200.so).

Surfaces mirroring the reference: ``ops`` (fastmd.ops), ``graph`` and ``line_graph`` (fastmd.graph
builders, the MatRIS bond pairs and triplets), ``wide_gemm`` and ``decomposed_indexed_cat_silu_linear``
(fastmd.engine.kernels), ``segment_attention``, ``gated_ln`` and ``pair_aggregate`` (the MatRIS receiver
attention, GatedMLP epilogue and directed-pair aggregation), ``energy_derivative``
(fastmd.engine), ``residual_add`` and ``dispatch`` (the MatRIS residual add and the ``OpDispatcher``
operator surface of the model sites), ``gpu_nhc``, ``whole_step``, ``model_graph`` and ``md_protocol`` (fastmd.execution /
fastmd.interfaces: the execution modes, restart files and extxyz frames), ``mace`` (the MACE-architecture
energy tap).
"""
from fastmd_b200 import (  # noqa: F401
    _lib, decomposed_indexed_cat_silu_linear, dispatch, energy_derivative, gated_ln, gpu_nhc, graph, line_graph, mace,
    md_protocol, model_graph, ops, pair_aggregate, residual_add, segment_attention, units, whole_step, wide_gemm)

__all__ = ["decomposed_indexed_cat_silu_linear", "dispatch", "energy_derivative", "gated_ln", "gpu_nhc", "graph",
           "line_graph", "mace", "md_protocol", "model_graph", "ops", "pair_aggregate", "residual_add",
           "segment_attention", "units", "whole_step", "wide_gemm"]
