"""CPU restatement of the reference's decomposed indexed-concat SiLU epilogue -- TEST INFRASTRUCTURE ONLY.

fastmd/engine/kernels/decomposed_indexed_cat_silu_linear.py, the epilogue after the projections
``p_k = X_k W_k^T`` ([rows_k, 2H], core half then gate half):

* forward ``_cat3_gather_add_silu_fwd`` (:97) / ``_cat4_gather_add_silu_fwd`` (:156):
  ``preact = p0 + p1[ia] + p2[ib] (+ p3[ic]) + bias``, added in that order in FP32, then
  ``core_act = core * sigmoid(core)`` and ``gate_act = gate * sigmoid(gate)`` with
  ``sigmoid(x) = 1 / (1 + exp(-x))``;
* backward ``_cat3_gather_add_silu_bwd`` (:234) / ``_cat4`` (:383): ``d = g * s * (1 + x (1 - s))`` per
  half, ``grad_p0 = [dcore | dgate]`` per row and ``grad_p_k[index_k[r]] += d[r]`` for the gathered parts.

Pinned against the reference kernels under TRITON_INTERPRET=1 (tests/golden/gather_add_silu.npz):
bitwise for preact, the activations and grad_p0; the scattered sums in row order (the reference's
deterministic ordered sum) agree with the kernels' atomic order to FP32 rounding.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _sigmoid(x):
    return F32(1) / (F32(1) + np.exp(-x))


def forward(p0, gathered, bias=None):
    """``gathered``: [(p_k [n_k, 2H], index_k [rows])...]; returns (preact, core_act, gate_act)."""
    pre = np.asarray(p0, F32).copy()
    for p, idx in gathered:
        pre = pre + np.asarray(p, F32)[np.asarray(idx)]
    if bias is not None:
        pre = pre + np.asarray(bias, F32)[None, :]
    H = pre.shape[1] // 2
    core, gate = pre[:, :H], pre[:, H:]
    return pre, core * _sigmoid(core), gate * _sigmoid(gate)


def silu_grad(x, g):
    s = _sigmoid(x)
    return g * s * (F32(1) + x * (F32(1) - s))


def backward(grad_core, grad_gate, preact, gathered_shapes):
    """(grad_p0 [rows, 2H], [grad_p_k [n_k, 2H]...]) with ``gathered_shapes`` [(n_k, index_k)...]."""
    pre = np.asarray(preact, F32)
    H = pre.shape[1] // 2
    d = np.concatenate([silu_grad(pre[:, :H], np.asarray(grad_core, F32)),
                        silu_grad(pre[:, H:], np.asarray(grad_gate, F32))], axis=1)
    grads = []
    for n, idx in gathered_shapes:
        g = np.zeros((n, 2 * H), F32)
        for r, i in enumerate(np.asarray(idx)):  # row order
            g[i] += d[r]
        grads.append(g)
    return d, grads
