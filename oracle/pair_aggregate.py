"""CPU restatement of the reference's directed-pair aggregation -- TEST INFRASTRUCTURE ONLY.

The MatRIS atom graph stores each undirected edge as two directed rows; ``pair_index[U, 2]`` names
them. The reference's kernels (fastmd/models/matris/op/triton_directed_pair_aggregate.py) compute, in
FP32:

* ``_directed_pair_average_fwd`` (:61): ``out[u] = (data[p0] + data[p1]) * 0.5``;
* ``_directed_pair_average_bwd`` (:83): ``grad[p0] = grad[p1] = gout[u] * 0.5``;
* ``_undirected_pair_expand_fwd`` (:105): ``out[p0] = out[p1] = data[u]``;
* ``_undirected_pair_expand_bwd`` (:127): ``grad[u] = gout[p0] + gout[p1]``.

Each output element is one FP32 addition and/or one multiplication by 0.5 (exact), so NumPy float32
arithmetic reproduces them to the bit. Pinned bitwise against the reference kernels run under
TRITON_INTERPRET=1 (tests/golden/pair_aggregate.npz, made by tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def average(data, pair):
    """[U, D] = (data[p0] + data[p1]) * 0.5 for data [2U, D] (any row stride)."""
    data = np.asarray(data, F32)
    pair = np.asarray(pair, np.int64)
    return ((data[pair[:, 0]] + data[pair[:, 1]]) * F32(0.5)).astype(F32)


def average_bwd(gout, pair, num_directed):
    """[2U, D]: each directed row of pair u receives gout[u] * 0.5."""
    gout = np.asarray(gout, F32)
    pair = np.asarray(pair, np.int64)
    out = np.zeros((num_directed, gout.shape[1]), F32)
    half = (gout * F32(0.5)).astype(F32)
    out[pair[:, 0]] = half
    out[pair[:, 1]] = half
    return out


def expand(data, pair, num_directed):
    """[2U, D]: both directed rows of pair u receive data[u]."""
    data = np.asarray(data, F32)
    pair = np.asarray(pair, np.int64)
    out = np.zeros((num_directed, data.shape[1]), F32)
    out[pair[:, 0]] = data
    out[pair[:, 1]] = data
    return out


def expand_bwd(gout, pair):
    """[U, D] = gout[p0] + gout[p1]."""
    gout = np.asarray(gout, F32)
    pair = np.asarray(pair, np.int64)
    return (gout[pair[:, 0]] + gout[pair[:, 1]]).astype(F32)
