"""CPU restatement of the reference's fixed-capacity MatRIS bond graph -- TEST INFRASTRUCTURE ONLY.

A builder with a line graph (fastmd/graph/fixed_capacity_builder.py) turns the per-step edges into
fixed-capacity rows of directed edges, undirected pairs and triplets:

* padding rows past the real edges: ``_pad_edges_kernel`` (:292; sink atoms: both rows of padded pair p
  on sink ``N + p n_dummy / n_pad_u``, image (3, 3, 3)) or ``_pad_loop_pairs_kernel`` (:397; far
  self-loops: padded pair p is the two opposite loops, images +image / -image, of atom p mod N);
* ``_materialize_pairs`` (:2001): the real rows in canonical key order, each row's reverse found by
  ``searchsorted`` of its reverse key, a pair leader where ``row <= reverse``, ``directed2undirected``
  the leader rank of ``min(row, reverse)`` (padded rows: padded pairs in order),
  ``undirected2directed`` the leader row (padded pairs: their first padded row), ``invalid_pairs`` on an
  odd count, a pair count unequal to half the edges, or a real row without its reverse;
* ``_materialize_line_graph`` (:2101) and ``_line_graph_kernel`` (:681): the short rows of each centre
  (``short_edge_matrix``), ``pair_offsets`` = scan of ``k (k - 1)``, triplet row
  ``[atom, u(first), first, u(second), second]`` with ``first = l // (k - 1)``, ``second`` skipping
  ``first``; padded triplets on padded pairs; ``overflow`` = edges >= e_capacity, triplets >
  t_capacity, invalid pairs or invalid candidates;
* ``_allocate_overflow_topology`` (:1474) and ``_substitute_overflow_topology`` (:2163): on overflow
  every row is replaced by the all-padding topology.

Pinned bitwise against those reference methods run on CPU (their Triton kernels under TRITON_INTERPRET=1)
in tests/golden/bond_graph.npz, made by tests/golden/make_golden.py.
"""
from __future__ import annotations

import numpy as np

MAX_IMAGE = 10


def _keys(center, neighbor, images, n_real, reverse=False):
    radix = 2 * MAX_IMAGE + 1
    c, n = np.asarray(center, np.int64), np.asarray(neighbor, np.int64)
    im = np.asarray(images, np.int64) * (-1 if reverse else 1)
    first, second = (n, c) if reverse else (c, n)
    return ((first * n_real + second) * radix**3 + (im[:, 0] + MAX_IMAGE) * radix * radix
            + (im[:, 1] + MAX_IMAGE) * radix + im[:, 2] + MAX_IMAGE)


def pad_rows(total, e_capacity, n_real, sink, n_dummy=0, pad_image=(0, 0, 0)):
    """(center, neighbor, images) of the padded rows ``[min(total, e_capacity), e_capacity)``."""
    tc = min(total, e_capacity)
    pad = np.arange(e_capacity - tc, dtype=np.int64)
    if sink:
        n_pad_u = e_capacity // 2 - tc // 2
        atom = n_real + (pad // 2) * n_dummy // max(n_pad_u, 1)
        images = np.full((pad.size, 3), 3, np.int64)
    else:
        atom = (pad // 2) % n_real
        sign = 1 - 2 * (pad % 2)
        images = sign[:, None] * np.asarray(pad_image, np.int64)[None, :]
    return atom, atom.copy(), images


def build(center, neighbor, images, short, total, *, n_real, u_capacity, t_capacity, sink, n_dummy=0,
          pad_image=(0, 0, 0), short_counts=None, candidate_valid=True):
    """The bond graph of the real edges ``(center, neighbor, images, short)`` (any order; ``total`` rows,
    the unclamped edge count; rows past the capacity are dropped as the reference's materialization
    drops them). Returns a dict of ``center``, ``neighbor``, ``images`` [E_cap(, 3)], ``d2u`` [E_cap],
    ``u2d`` [U_cap], ``line_graph`` [T_cap, 5], ``overflow``, ``invalid_pairs``, ``n_triplets``."""
    e_cap = 2 * u_capacity
    N = n_real
    tc = min(total, e_cap)
    center = np.asarray(center, np.int64)[:tc]
    neighbor = np.asarray(neighbor, np.int64)[:tc]
    images = np.asarray(images, np.int64)[:tc]
    short = np.asarray(short, bool)[:tc]
    if short_counts is None:
        short_counts = np.bincount(center[short], minlength=N).astype(np.int64)
    pc, pn, pi = pad_rows(total, e_cap, N, sink, n_dummy, pad_image)
    C, Nb, Im = np.concatenate([center, pc]), np.concatenate([neighbor, pn]), np.concatenate([images, pi])
    S = np.concatenate([short, np.zeros(pc.size, bool)])
    ids = np.arange(e_cap, dtype=np.int64)
    real = ids < tc
    invalid_key = np.iinfo(np.int64).max - e_cap + ids
    # _materialize_pairs: canonical order, reverse search, leaders
    fwd = np.where(real, _keys(C, Nb, Im, N), invalid_key)
    order = np.argsort(fwd, kind="stable")
    sorted_key = fwd[order]
    C, Nb, Im, S = C[order], Nb[order], Im[order], S[order]
    rev = np.where(real, _keys(C, Nb, Im, N, reverse=True), invalid_key)
    pos = np.minimum(np.searchsorted(sorted_key, rev, side="left"), e_cap - 1)
    match = sorted_key[pos] == rev
    leader = real & match & (ids <= pos)
    prefix = np.cumsum(leader.astype(np.int64))
    real_pair = prefix[np.minimum(ids, pos)] - 1
    real_u = tc // 2
    d2u = np.clip(np.where(real, real_pair, real_u + np.maximum(ids - tc, 0) // 2), 0, u_capacity - 1)
    scatter = np.full(u_capacity + e_cap, e_cap, np.int64)
    target = np.where(leader, np.clip(real_pair, 0, u_capacity), u_capacity + ids)
    np.minimum.at(scatter, target, ids)
    u_ids = np.arange(u_capacity, dtype=np.int64)
    u2d = np.minimum(np.where(u_ids < real_u, scatter[:u_capacity], tc + 2 * np.maximum(u_ids - real_u, 0)),
                     e_cap - 1)
    invalid = bool(total % 2 != 0 or leader.sum() != total // 2 or np.any(real & ~match))
    # _materialize_line_graph: short rows per centre, triplet numbering
    is_short = real & S
    safe_c = np.clip(C, 0, N - 1)
    # short_edge_matrix[a, l] = the l-th short row of a (one row per short edge, no slot limit here)
    short_rows = {}
    for e in np.nonzero(is_short)[0]:
        short_rows.setdefault(int(safe_c[e]), []).append(int(e))
    pair_counts = short_counts * (short_counts - 1)
    pair_off = np.concatenate([[0], np.cumsum(pair_counts)])
    n_trip = int(pair_off[-1])
    overflow = bool(total >= e_cap or n_trip > t_capacity or invalid or not candidate_valid)
    t_ids = np.arange(t_capacity, dtype=np.int64)
    if overflow:
        safe_u = ids // 2
        o_center = N + safe_u * n_dummy // u_capacity if sink else safe_u % N
        sign = np.where(ids % 2 == 0, 1, -1)
        o_img = sign[:, None] * (np.full(3, 3) if sink else np.asarray(pad_image, np.int64))[None, :]
        if sink:
            line_u = ((t_ids * n_dummy // t_capacity) * u_capacity + n_dummy - 1) // n_dummy
        else:
            line_u = t_ids * u_capacity // t_capacity
        line_u = np.minimum(line_u, u_capacity - 1)
        line_de = 2 * line_u
        lg = np.stack([o_center[line_de], line_u, line_de, line_u, line_de], 1)
        return dict(center=o_center, neighbor=o_center.copy(), images=o_img, d2u=safe_u, u2d=2 * u_ids,
                    line_graph=lg, overflow=True, invalid_pairs=invalid, n_triplets=n_trip)
    t_clamped = min(n_trip, t_capacity)
    lg = np.zeros((t_capacity, 5), np.int64)
    for t in range(t_clamped):
        atom = int(np.searchsorted(pair_off, t, side="right") - 1)
        local = t - pair_off[atom]
        k = int(short_counts[atom])
        denom = max(k - 1, 1)
        first = local // denom
        second_raw = local - first * denom
        second = second_raw + int(second_raw >= first)
        e1, e2 = short_rows[atom][first], short_rows[atom][second]
        lg[t] = (atom, d2u[e1], e1, d2u[e2], e2)
    pad_id = np.maximum(t_ids[t_clamped:] - t_clamped, 0)
    pad_pair = pad_id % max(u_capacity - real_u, 1)
    pad_u = real_u + pad_pair
    pad_de = tc + 2 * pad_pair
    pad_atom = N + pad_id * n_dummy // max(t_capacity - t_clamped, 1) if sink else pad_pair % N
    lg[t_clamped:] = np.stack([pad_atom, pad_u, pad_de, pad_u, pad_de], 1)
    return dict(center=C, neighbor=Nb, images=Im, d2u=d2u, u2d=u2d, line_graph=lg, overflow=False,
                invalid_pairs=invalid, n_triplets=n_trip)
