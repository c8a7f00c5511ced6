"""CPU restatement of the reference's MatRIS residual add -- TEST INFRASTRUCTURE ONLY.

``out = delta + residual * weight[None, :]`` and its backward ``grad_residual = gout * weight[None, :]``
(``grad_delta = gout``) in FP32, the product rounded before the addition, as
fastmd/models/matris/op/triton_residual_add.py:40 (``_residual_add_fwd``) and :64
(``_residual_add_bwd``) compute them.

Pinned against the reference kernels run under TRITON_INTERPRET=1 (tests/golden/residual_add.npz, made by
tests/golden/make_golden.py): bitwise.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def forward(delta, residual, weight):
    """[N, D] float32; ``weight`` [D] (any shape with D elements)."""
    w = np.asarray(weight, F32).reshape(1, -1)
    return (np.asarray(delta, F32) + np.asarray(residual, F32) * w).astype(F32)


def backward(gout, weight):
    """(grad_delta, grad_residual) of ``forward``; the frozen weight has no gradient."""
    g = np.asarray(gout, F32)
    return g, (g * np.asarray(weight, F32).reshape(1, -1)).astype(F32)
