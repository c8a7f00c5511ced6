"""CPU restatement of the MatRIS reverse-edge pairing and line graph -- TEST INFRASTRUCTURE ONLY.

fastmd/graph/gpu_graph_builder.py:
* ``_build_d2u`` (:217): forward key ``(c N + n) V + code(image)`` and reverse key
  ``(n N + c) V + code(-image)`` (``V = (2 M + 1)^3``, ``code`` in radix ``2 M + 1`` with offset
  ``M = MAX_IMAGE = 10``); ``pair(e)`` = the position of ``e``'s reverse key among the sorted forward
  keys (clamped to the last edge; through the sort permutation unless presorted);
  ``directed2undirected(e)`` = the rank of ``min(e, pair(e))`` among the distinct such minima and
  ``undirected2directed(u)`` = the smallest edge of undirected edge ``u``;
* ``_build_line_graph`` (:511): the short edges (``dist < cutoff``) grouped by centre in a stable
  order; for an atom with ``k`` of them the ``k (k - 1)`` ordered pairs ``(first, second)``,
  ``first = l // (k - 1)``, ``second = l % (k - 1)`` skipping ``first``; rows
  ``[atom, u(first), e(first), u(second), e(second)]`` int32.

Pinned bitwise against the reference's functions run in this container
(tests/golden/line_graph.npz).
"""
from __future__ import annotations

import numpy as np

MAX_IMAGE = 10


def _keys(center, neighbor, images, n_atoms, max_image=MAX_IMAGE):
    radix = 2 * max_image + 1
    volume = radix ** 3
    c, n, img = (np.asarray(x, np.int64) for x in (center, neighbor, images))
    fwd = (c * n_atoms + n) * volume + (img[:, 0] + max_image) * radix * radix + (img[:, 1] + max_image) * radix \
        + (img[:, 2] + max_image)
    rev = (n * n_atoms + c) * volume + (-img[:, 0] + max_image) * radix * radix + (-img[:, 1] + max_image) * radix \
        + (-img[:, 2] + max_image)
    return fwd, rev


def build_d2u(center, neighbor, images, n_atoms, presorted=False):
    """(directed2undirected [E] int32, undirected2directed [U] int32)."""
    E = len(center)
    if E == 0:
        return np.zeros(0, np.int32), np.zeros(0, np.int32)
    fwd, rev = _keys(center, neighbor, images, n_atoms)
    if presorted:
        pair = np.minimum(np.searchsorted(fwd, rev, side="left"), E - 1)
    else:
        order = np.argsort(fwd, kind="stable")
        pos = np.minimum(np.searchsorted(fwd[order], rev, side="left"), E - 1)
        pair = order[pos]
    mins = np.minimum(np.arange(E), pair)
    uvals, d2u = np.unique(mins, return_inverse=True)
    u2d = np.full(len(uvals), E, np.int64)
    np.minimum.at(u2d, d2u, np.arange(E))
    return d2u.astype(np.int32), u2d.astype(np.int32)


def build_line_graph(center, d2u, dist, n_atoms, cutoff, presorted=False):
    """Triplets [T, 5] int32."""
    center = np.asarray(center, np.int64)
    short = np.nonzero(np.asarray(dist, np.float32) < np.float32(cutoff))[0]
    if len(short) == 0:
        return np.zeros((0, 5), np.int32)
    if not presorted:
        short = short[np.argsort(center[short], kind="stable")]
    sc = center[short]
    counts = np.bincount(sc, minlength=n_atoms).astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]])
    rows = []
    for atom in range(n_atoms):
        k = counts[atom]
        for local in range(k * (k - 1)):
            first = local // (k - 1)
            second_raw = local % (k - 1)
            second = second_raw + (second_raw >= first)
            e1, e2 = short[offsets[atom] + first], short[offsets[atom] + second]
            rows.append((atom, d2u[e1], e1, d2u[e2], e2))
    return np.asarray(rows, np.int32).reshape(-1, 5)
