"""fastmd_b200: FastMD's per-step MD hot path on hand-written sm_100a kernels (libfastmd_b200.so).

Surfaces mirroring the reference: ``ops`` (fastmd.ops), ``graph`` and ``line_graph`` (fastmd.graph
builders, the MatRIS bond pairs and triplets), ``wide_gemm`` and ``decomposed_indexed_cat_silu_linear``
(fastmd.engine.kernels), ``segment_attention``, ``gated_ln``, ``pair_aggregate`` and ``residual_add`` (the
MatRIS receiver attention, GatedMLP epilogue, directed-pair aggregation and residual add), ``dispatch``
(the ``OpDispatcher`` operator surface of the model sites), ``energy_derivative`` (fastmd.engine),
``gpu_nhc``, ``whole_step``, ``model_graph``, ``skin_topology`` and ``md_protocol`` (fastmd.execution /
fastmd.interfaces: the execution modes, the calculator's skin-epoch topology reuse, restart files and
extxyz frames), ``mace`` (the MACE-architecture energy tap), ``nequip`` (the NequIP-architecture,
SevenNet-0-style potential of config 3).
"""
from fastmd_b200 import (  # noqa: F401
    _lib, decomposed_indexed_cat_silu_linear, dispatch, energy_derivative, gated_ln, gpu_nhc, graph, line_graph, mace,
    md_protocol, model_graph, nequip, ops, pair_aggregate, residual_add, segment_attention, skin_topology, units, whole_step,
    wide_gemm)

__all__ = ["decomposed_indexed_cat_silu_linear", "dispatch", "energy_derivative", "gated_ln", "gpu_nhc", "graph",
           "line_graph", "mace", "md_protocol", "model_graph", "nequip", "ops", "pair_aggregate", "residual_add",
           "segment_attention", "skin_topology", "units", "whole_step", "wide_gemm"]
