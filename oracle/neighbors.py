"""NumPy restatements of FastMD's neighbour-list arithmetic -- test oracle.

* ``small_matmul``: fastmd/graph/geometry.py:7 (``(a[..., :, None] * b).sum(-2)``
  in float32, summed left to right).
* ``wrap``: the build prologue of fastmd/graph/fixed_capacity_builder.py:2203-2208
  (frac = pos @ inv(cell), wraps = floor(frac), wrapped = (frac - wraps) @ cell).
* ``refilter``: the per-step exact re-filter of a candidate list,
  ``_count_neighbors_kernel`` / ``_materialize_neighbors_kernel``
  (fixed_capacity_builder.py:98 / :189; arithmetic :159-163): float32
  ``dx = nx - px + sx*c0 + sy*c3 + sz*c6`` evaluated left to right,
  ``dist2 = dx*dx + dy*dy + dz*dz``, edge iff ``dist2 < rc*rc``.
* ``ragged_filter``: the eager path's re-filter (fastmd/graph/gpu_graph_builder.py:186-192):
  ``diff = (pos[n] - pos[c]) + img @ cell``, ``dist = |diff|``, edge iff ``dist < rc``.
* ``sort_key``: the canonical (centre, neighbour, image) key
  (fixed_capacity_builder.py:1978-1996; gpu_graph_builder.py:199-210).
* ``dense_pairs``: the FP64 O(N^2 x images) search of the reference's
  boundary tests (tests/test_fixed_capacity_boundary.py:86-103).
* ``far_loop_image`` / ``pad_self_loops``: far self-loop padding
  (fixed_capacity_builder.py:1006-1027 and ``_pad_self_loops_kernel`` :324).
* ``candidates``: a full candidate list within ``cutoff`` (FP64 distance), the
  role nvalchemiops' cell-list query plays in the reference (its exact tie rule
  never decides an edge: the re-filter does).
"""
from __future__ import annotations

import math

import numpy as np

f32 = np.float32


def small_matmul(a, b):
    a = np.asarray(a, dtype=f32)
    b = np.asarray(b, dtype=f32)
    prod = a[..., :, None] * b[None, :, :]          # [rows, k, cols], float32
    out = prod[..., 0, :]
    for k in range(1, prod.shape[-2]):
        out = (out + prod[..., k, :]).astype(f32)
    return out.astype(f32)


def inverse_cell(cell):
    """float32 inverse of the cell: the float64 inverse rounded once."""
    return np.linalg.inv(np.asarray(cell, dtype=np.float64)).astype(f32)


def wrap(positions, cell, inv_cell=None):
    inv_cell = inverse_cell(cell) if inv_cell is None else np.asarray(inv_cell, f32)
    frac_un = small_matmul(positions, inv_cell)
    wraps = np.floor(frac_un).astype(np.int32)
    frac = (frac_un - wraps.astype(f32)).astype(f32)
    return small_matmul(frac, cell), wraps, frac


def refilter(wrapped, cell, cand_matrix, cand_shifts, cand_count, cutoff, wrap_delta=None, line_cutoff=None):
    """Edges of a candidate list in candidate order: (center, neighbor, image int32 [E,3], dist f32), and
    with ``line_cutoff`` the short flags ``dist2 < line_cutoff**2`` of the same float32 ``dist2``
    (``_materialize_neighbors_kernel``'s ``short_valid``, fixed_capacity_builder.py:264)."""
    wrapped = np.asarray(wrapped, f32)
    cell = np.asarray(cell, f32)
    n, bmax = cand_matrix.shape
    wd = np.zeros((n, 3), np.int32) if wrap_delta is None else np.asarray(wrap_delta, np.int32)
    cut2 = f32(cutoff * cutoff)
    centers, neighbors, images, dists, shorts = [], [], [], [], []
    line2 = None if line_cutoff is None else f32(line_cutoff * line_cutoff)
    for atom in range(n):
        cnt = int(cand_count[atom])
        nb = np.minimum(cand_matrix[atom, :cnt].astype(np.int64), n - 1)
        s = cand_shifts[atom, :cnt].astype(np.int32) + wd[nb] - wd[atom]
        sf = s.astype(f32)
        p = wrapped[atom]
        q = wrapped[nb]
        d = []
        for axis in range(3):
            v = (q[:, axis] - p[axis]).astype(f32)
            v = (v + sf[:, 0] * cell[0, axis]).astype(f32)
            v = (v + sf[:, 1] * cell[1, axis]).astype(f32)
            v = (v + sf[:, 2] * cell[2, axis]).astype(f32)
            d.append(v)
        dist2 = ((d[0] * d[0] + d[1] * d[1]).astype(f32) + d[2] * d[2]).astype(f32)
        keep = dist2 < cut2
        centers.append(np.full(int(keep.sum()), atom, np.int64))
        neighbors.append(nb[keep])
        images.append(s[keep])
        dists.append(np.sqrt(dist2[keep]).astype(f32))
        if line2 is not None:
            shorts.append(dist2[keep] < line2)
    out = (np.concatenate(centers), np.concatenate(neighbors), np.concatenate(images).reshape(-1, 3),
           np.concatenate(dists))
    return out if line2 is None else (*out, np.concatenate(shorts))


def ragged_filter(wrapped, cell, center, neighbor, images, cutoff):
    wrapped = np.asarray(wrapped, f32)
    diff = (wrapped[neighbor] - wrapped[center]).astype(f32)
    diff = (diff + small_matmul(images.astype(f32), cell)).astype(f32)
    dist = np.sqrt(((diff[:, 0] * diff[:, 0] + diff[:, 1] * diff[:, 1]).astype(f32)
                    + diff[:, 2] * diff[:, 2]).astype(f32))
    return dist < f32(cutoff), dist


def sort_key(center, neighbor, images, n_atoms, max_image=10):
    radix = 2 * max_image + 1
    images = np.asarray(images, np.int64)
    return ((np.asarray(center, np.int64) * n_atoms + np.asarray(neighbor, np.int64)) * radix**3
            + (images[:, 0] + max_image) * radix * radix + (images[:, 1] + max_image) * radix
            + images[:, 2] + max_image)


def canonical(center, neighbor, images, n_atoms, *extra):
    order = np.argsort(sort_key(center, neighbor, images, n_atoms), kind="stable")
    return (center[order], neighbor[order], images[order], *[e[order] for e in extra])


def heights(cell):
    cell = np.asarray(cell, np.float64)
    vol = abs(np.linalg.det(cell))
    return vol / np.array([np.linalg.norm(np.cross(cell[(k + 1) % 3], cell[(k + 2) % 3])) for k in range(3)])


def dense_pairs(wrapped, cell, cutoff):
    """{(i, j, nx, ny, nz): distance} of every directed pair within ``cutoff`` (FP64)."""
    pos = np.asarray(wrapped, np.float64)
    cell = np.asarray(cell, np.float64)
    reach = [int(np.ceil(cutoff / h)) + 1 for h in heights(cell)]
    pairs = {}
    for ix in range(-reach[0], reach[0] + 1):
        for iy in range(-reach[1], reach[1] + 1):
            for iz in range(-reach[2], reach[2] + 1):
                shift = np.array([ix, iy, iz], np.float64) @ cell
                d = np.linalg.norm(pos[None, :, :] + shift - pos[:, None, :], axis=-1)
                for i, j in zip(*np.nonzero(d < cutoff)):
                    if i != j or (ix, iy, iz) != (0, 0, 0):
                        pairs[(int(i), int(j), ix, iy, iz)] = float(d[i, j])
    return pairs


def candidates(wrapped, cell, cutoff, bmax=None):
    """Full candidate matrix (neighbour [N, B] int32 filled with N, shifts [N, B, 3], counts [N])."""
    pairs = dense_pairs(wrapped, cell, cutoff)
    n = np.asarray(wrapped).shape[0]
    rows = [[] for _ in range(n)]
    for (i, j, ix, iy, iz) in sorted(pairs):
        rows[i].append((j, ix, iy, iz))
    width = max([len(r) for r in rows] + [1]) if bmax is None else bmax
    nm = np.full((n, width), n, np.int32)
    ns = np.zeros((n, width, 3), np.int32)
    nn = np.zeros(n, np.int32)
    for i, r in enumerate(rows):
        nn[i] = len(r)
        for k, (j, ix, iy, iz) in enumerate(r[:width]):
            nm[i, k] = j
            ns[i, k] = (ix, iy, iz)
    return nm, ns, nn


def far_loop_image(cell, cutoff, min_length=0.0):
    """(image, length): a whole number of the longest lattice vector, >= 2 cutoff."""
    lengths = np.linalg.norm(np.asarray(cell, np.float64), axis=1)
    axis = int(np.argmax(lengths))
    multiple = max(1, math.ceil(max(min_length, 2.0 * cutoff) / lengths[axis]))
    image = [0, 0, 0]
    image[axis] = multiple
    return tuple(image), multiple * float(lengths[axis])


def pad_self_loops(n_edges, e_capacity, n_atoms, image):
    """Padded rows [n_edges, e_capacity): loops of atom k mod N with the far image."""
    k = np.arange(max(e_capacity - n_edges, 0))
    atoms = k % n_atoms
    return atoms, atoms, np.tile(np.asarray(image, np.int32), (k.size, 1))


def estimate_max_neighbors(cutoff, atomic_density=0.35, safety_factor=5.0):
    """fastmd/graph/neighbor_list_backend.py:77 (per-atom candidate slots, multiple of 16)."""
    if cutoff <= 0:
        return 0
    expected = max(1, safety_factor * atomic_density * (4.0 / 3.0) * math.pi * cutoff**3)
    return int(math.ceil(expected / 16)) * 16


def float64_prologue(positions64, cell64, reference32, reference_wraps, skin, inv_cell=None):
    """The float64 build's prologue (``_float64_prologue_kernel``, fixed_capacity_builder.py:464):
    the float32 wrap of the rounded coordinates ``q`` (``wrap``), the float64 model positions
    ``p - ((w0 c[0] + w1 c[1]) + w2 c[2])`` (the same whole lattice vectors of the float64 cell),
    the wrap delta against the refresh, the largest float32 displacement ``q - reference`` and the
    skin test ``2 max <= skin + 1e-6``. Returns a dict of those arrays."""
    p = np.asarray(positions64, np.float64)
    c64 = np.asarray(cell64, np.float64)
    q = p.astype(f32)
    wrapped, wraps, frac = wrap(q, c64.astype(f32), inv_cell)
    v = wraps.astype(np.float64)
    model = p - ((v[:, 0:1] * c64[0] + v[:, 1:2] * c64[1]) + v[:, 2:3] * c64[2])
    d = (q - np.asarray(reference32, f32)).astype(f32)
    dd = ((d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]).astype(f32) + d[:, 2] * d[:, 2]).astype(f32)
    largest = np.sqrt(dd.max(initial=f32(0))).astype(f32)
    return {"wrapped": wrapped, "frac": frac, "model_positions": model,
            "wrap_delta": (wraps - np.asarray(reference_wraps, np.int32)).astype(np.int32),
            "max_displacement": largest, "candidate_valid": bool(largest * f32(2) <= f32(skin + 1.0e-6))}


def pad_vector_override(n_edges, e_capacity, vector):
    """The edge-vector override of exact-rc loop padding (``_pad_self_loops_kernel`` with
    ``HAS_OVERRIDE``, fixed_capacity_builder.py:324): ``vector`` on rows ``>= min(n_edges, e_capacity)``,
    0 on the real rows; [e_capacity, 3] float32."""
    out = np.zeros((e_capacity, 3), f32)
    out[min(n_edges, e_capacity):] = np.asarray(vector, f32)
    return out
