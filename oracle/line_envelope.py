"""CPU restatement of the MatRIS line-graph envelope product -- TEST INFRASTRUCTURE ONLY.

``env[t] = base[source[t]] * base[target[t]]`` (float32) and its backward, each triplet adding
``gout[t] * base[target[t]]`` to its source bond's gradient row and ``gout[t] * base[source[t]]`` to its
target bond's, in blocks of 16 triplets (a block's source side, then its target side): the arithmetic of fastmd/models/matris/op/triton_line_envelope.py:50
(``_line_envelope_fwd``) and :87 (``_line_envelope_bwd``, whose float atomics the interpreter applies in
this order). Pinned against those kernels run under TRITON_INTERPRET=1 (tests/golden/line_envelope.npz):
bitwise.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def forward(base, source, target):
    base = np.asarray(base, F32)
    return (base[np.asarray(source)] * base[np.asarray(target)]).astype(F32)


def backward(gout, base, source, target, block=16):
    """Rows in blocks of ``block`` (the kernel's BM): a block's source-side additions, then its target
    side's, row by row (the order the interpreter applies a block's atomics in)."""
    base, gout = np.asarray(base, F32), np.asarray(gout, F32)
    source, target = np.asarray(source), np.asarray(target)
    grad = np.zeros_like(base)
    for start in range(0, len(source), block):
        rows = range(start, min(start + block, len(source)))
        for t in rows:
            grad[source[t]] = (grad[source[t]] + gout[t] * base[target[t]]).astype(F32)
        for t in rows:
            grad[target[t]] = (grad[target[t]] + gout[t] * base[source[t]]).astype(F32)
    return grad
