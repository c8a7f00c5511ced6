"""NumPy restatements of the reference's edge/node operators -- test oracle.

* ``aligned_gather_cat3``: fastmd/models/matris/op/triton_gather_cat.py:30
  (forward) and :59 (backward: grad of the aligned block is a copy, the
  gathered rows receive the scatter-add of their output blocks).
* ``aligned_gather_cat4``: triton_gather_cat.py:203 / :236.
* ``csr_segment_sum``: fastmd/models/matris/op/triton_csr_segment_sum.py:71
  (out[s] = sum over the CSR run of s of weight * value), VJP :184
  (gvalue = gout[seg] * weight, gweight = gout[seg] * value).
* ``segment_csr``: segment_attention_csr_metadata
  (fastmd/models/matris/op/triton_segment_attention.py:824): stable argsort of
  the segments and their run offsets.

Sums are accumulated in float64 and rounded once (the reference's FP32 tile
order is not reproduced; float comparisons use a tolerance).
"""
from __future__ import annotations

import numpy as np


def aligned_gather_cat3(aligned, gathered, index_a, index_b):
    return np.concatenate([aligned, gathered[index_a], gathered[index_b]], axis=1)


def aligned_gather_cat3_bwd(gout, n_gathered, index_a, index_b):
    dim = gout.shape[1] // 3
    grad_aligned = gout[:, :dim].copy()
    acc = np.zeros((n_gathered, dim), dtype=np.float64)
    np.add.at(acc, index_a, gout[:, dim:2 * dim].astype(np.float64))
    np.add.at(acc, index_b, gout[:, 2 * dim:].astype(np.float64))
    return grad_aligned, acc.astype(gout.dtype)


def aligned_gather_cat4(aligned, gathered_a, index_a, gathered_b, index_b, index_c):
    return np.concatenate([aligned, gathered_a[index_a], gathered_b[index_b], gathered_b[index_c]], axis=1)


def aligned_gather_cat4_bwd(gout, n_a, n_b, index_a, index_b, index_c):
    dim = gout.shape[1] // 4
    grad_aligned = gout[:, :dim].copy()
    ga = np.zeros((n_a, dim), dtype=np.float64)
    gb = np.zeros((n_b, dim), dtype=np.float64)
    np.add.at(ga, index_a, gout[:, dim:2 * dim].astype(np.float64))
    np.add.at(gb, index_b, gout[:, 2 * dim:3 * dim].astype(np.float64))
    np.add.at(gb, index_c, gout[:, 3 * dim:].astype(np.float64))
    return grad_aligned, ga.astype(gout.dtype), gb.astype(gout.dtype)


def gather_cat(parts, rows):
    """Mixed-width gather-cat: ``parts`` = [(src, index or None)]."""
    blocks = [src[:rows] if index is None else src[index] for src, index in parts]
    return np.concatenate(blocks, axis=1)


def segment_csr(segment, num_segment):
    """(perm, off): rows grouped by segment, ascending row order in a run."""
    segment = np.asarray(segment, dtype=np.int64)
    perm = np.argsort(segment, kind="stable")
    off = np.searchsorted(segment[perm], np.arange(num_segment + 1), side="left")
    return perm.astype(np.int64), off.astype(np.int64)


def csr_segment_sum(value, num_segment, perm, off, weight=None, skip_segment=-1):
    rows = value.astype(np.float64) if weight is None else weight.astype(np.float64) * value.astype(np.float64)
    out = np.zeros((num_segment, value.shape[1]), dtype=np.float64)
    for s in range(num_segment):
        if s == skip_segment:
            continue
        idx = perm[off[s]:off[s + 1]] if perm is not None else np.arange(off[s], off[s + 1])
        if idx.size:
            out[s] = rows[idx].sum(axis=0)
    return out.astype(value.dtype)


def segment_sum(value, segment, num_segment, weight=None, skip_segment=-1):
    """index_add_ form (fastmd/engine/kernels/segment.py:97 aggregate, average=False)."""
    rows = value.astype(np.float64) if weight is None else weight.astype(np.float64) * value.astype(np.float64)
    if skip_segment >= 0:
        rows = np.where((segment == skip_segment)[:, None], 0.0, rows)
    out = np.zeros((num_segment, value.shape[1]), dtype=np.float64)
    np.add.at(out, segment, rows)
    return out.astype(value.dtype)


def csr_segment_sum_bwd(gout, value, segment, weight=None, skip_segment=-1):
    g = gout[segment]
    if skip_segment >= 0:
        g = np.where((segment == skip_segment)[:, None], 0.0, g).astype(gout.dtype)
    gvalue = g if weight is None else (g * weight).astype(gout.dtype)
    gweight = (g * value).astype(gout.dtype)
    return gvalue, gweight
