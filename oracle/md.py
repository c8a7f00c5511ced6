"""CPU MD step of the hot path (neighbour list -> MACE-architecture forces -> NHC) -- test oracle.

The eager CPU path the reference runs for its config 0 (a CPU neighbour list,
the model's forward and backward, the torch NHC backend: gpu_nhc.py:1165-1195)
restated with this package's pieces: ``oracle.neighbors`` (the wrap prologue
and a dense FP64 search within the cutoff), ``oracle.mace`` (FP64 model and
autograd forces) and ``oracle.nhc`` (the NHC step in ASE's operation order,
float32 kick for float32 forces). Used as the checker of the GPU trajectory
and as the timed CPU baseline of bench.py.
"""
from __future__ import annotations

import numpy as np

from oracle import mace as omace
from oracle import neighbors as onb
from oracle import nhc as onhc


class OracleMD:
    def __init__(self, weights, config, positions, cell, numbers, masses, momenta, *, temperature_K, timestep,
                 tdamp, tchain=3, tloop=1):
        self.w, self.config = weights, config
        self.cell = np.asarray(cell, np.float64)
        self.cell32 = self.cell.astype(np.float32)
        self.inv32 = onb.inverse_cell(self.cell32)
        self.numbers = np.asarray(numbers)
        f, e = self.forces(np.asarray(positions, np.float64))
        self.nhc = onhc.NHC(masses, positions, momenta, f, temperature_K=temperature_K, timestep=timestep,
                            tdamp=tdamp, tchain=tchain, tloop=tloop, f32_kick=True, energy=e)

    def graph(self, positions):
        wrapped, _, _ = onb.wrap(np.asarray(positions, np.float32), self.cell32, inv_cell=self.inv32)
        pairs = onb.dense_pairs(wrapped, self.cell, self.config.r_max)
        keys = sorted(pairs)
        edges = np.array([k[:2] for k in keys], np.int64).reshape(-1, 2)
        images = np.array([k[2:] for k in keys], np.float64).reshape(-1, 3)
        return wrapped, edges, images

    def forces(self, positions):
        wrapped, edges, images = self.graph(positions)
        energy, forces, _ = omace.energy_forces(self.w, self.config, wrapped.astype(np.float64), self.cell,
                                                self.numbers, edges, images)
        return forces.astype(np.float32), float(energy[0])

    def step(self):
        q = self.nhc.pre_force()
        f, e = self.forces(q)
        self.nhc.post_force(f, e)
        return self.nhc


class MatRISOracleMD(OracleMD):
    """The same CPU MD step with the FP64 MatRIS oracle (``oracle.matris``): edges of a dense FP64 search
    within the atom cutoff, the bond pairing and triplets of ``oracle.line_graph`` (the reference's
    ``_build_d2u`` / ``_build_line_graph``), forces by autograd."""

    def __init__(self, params, config, positions, cell, numbers, masses, momenta, **kw):
        self.params = params
        super().__init__(None, config, positions, cell, numbers, masses, momenta, **kw)

    def graph(self, positions):
        from oracle import line_graph as olg

        wrapped, _, _ = onb.wrap(np.asarray(positions, np.float32), self.cell32, inv_cell=self.inv32)
        pairs = onb.dense_pairs(wrapped, self.cell, self.config.pairwise_cutoff)
        keys = sorted(pairs)
        edges = np.array([k[:2] for k in keys], np.int64).reshape(-1, 2)
        images = np.array([k[2:] for k in keys], np.int64).reshape(-1, 3)
        dist = np.array([pairs[k] for k in keys])
        d2u, u2d = olg.build_d2u(edges[:, 0], edges[:, 1], images, len(wrapped), presorted=True)
        lines = olg.build_line_graph(edges[:, 0], d2u, dist, len(wrapped), self.config.three_body_cutoff,
                                     presorted=True)
        return wrapped, edges, images, d2u, u2d, lines

    def forces(self, positions):
        from oracle import matris as om

        wrapped, edges, images, d2u, u2d, lines = self.graph(positions)
        energy, forces, _ = om.energy_forces_stress(self.params, self.config, wrapped.astype(np.float64), self.cell,
                                                    self.numbers, edges, images.astype(np.float64), d2u, u2d, lines)
        return forces.astype(np.float32), float(energy)
