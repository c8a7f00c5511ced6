"""Synthetic systems of the benchmark configurations (seeded; no dataset involved).

* ``perovskite``: the 3x3x3 cubic ABX3 supercell of BASELINE configs 0/1/4 -- a = 6.2 A,
  Cs (0,0,0), Sn (1/2,1/2,1/2), I at the three face centres, positions jittered by
  N(0, 0.05 A) from ``np.random.default_rng(seed)``, masses 132.905 / 118.71 / 126.904 amu.
* ``random_box``: N atoms uniform in a periodic cube of the given density (config 2).
"""
from __future__ import annotations

import numpy as np

SYMBOL_Z = {"Cs": 55, "Sn": 50, "I": 53}
MASSES = {55: 132.905, 50: 118.71, 53: 126.904}


def perovskite(reps: int = 3, a: float = 6.2, jitter: float = 0.05, seed: int = 0):
    """(positions [N,3] float64, cell [3,3], atomic numbers [N], masses [N])."""
    basis = np.array([[0.0, 0.0, 0.0], [0.5, 0.5, 0.5], [0.5, 0.5, 0.0], [0.5, 0.0, 0.5], [0.0, 0.5, 0.5]])
    numbers_cell = np.array([55, 50, 53, 53, 53])
    grid = np.array([[i, j, k] for i in range(reps) for j in range(reps) for k in range(reps)], dtype=np.float64)
    frac = (grid[:, None, :] + basis[None, :, :]).reshape(-1, 3)
    cell = np.eye(3) * (a * reps)
    positions = frac * a
    rng = np.random.default_rng(seed)
    positions = positions + rng.normal(0.0, jitter, positions.shape)
    numbers = np.tile(numbers_cell, len(grid))
    masses = np.array([MASSES[z] for z in numbers])
    return positions, cell, numbers, masses


def random_box(n_atoms: int = 100_000, density: float = 0.06, seed: int = 2, z: int = 14):
    """(positions, cell, atomic numbers) of ``n_atoms`` uniform in a cube of ``density`` atoms/A^3."""
    length = (n_atoms / density) ** (1.0 / 3.0)
    rng = np.random.default_rng(seed)
    positions = rng.uniform(0.0, length, (n_atoms, 3))
    return positions, np.eye(3) * length, np.full(n_atoms, z)
