"""NumPy restatement of FastMD's Nose-Hoover-chain step (ASE 3.29 NoseHooverChainNVT) -- test oracle.

* ``nhc_constants``: fastmd/execution/gpu_nhc.py:113 (kT, Q, 3N kT, the
  Suzuki-Yoshida sub-step table :90-94, the device constants layout, Q at
  index 16, gpu_nhc.py:273-275).
* ``maxwell_boltzmann_momenta``: gpu_nhc.py:199 (xi = default_rng(seed)
  .standard_normal((N, 3)); p = xi * sqrt(m kB T)).
* ``NHC.pre_force`` / ``NHC.post_force``: gpu_nhc.py:360 / :394 with the
  chain half step ``_nhc_half`` :333 and ``_p_eta_j`` :316, in the same
  operation order (one NumPy scalar/array op per rounding).
"""
from __future__ import annotations

import numpy as np

from oracle import units

FOURTH_ORDER_COEFFS = [
    1 / (2 - 2 ** (1 / 3)),
    -(2 ** (1 / 3)) / (2 - 2 ** (1 / 3)),
    1 / (2 - 2 ** (1 / 3)),
]
C_Q = 16


def nhc_constants(n_atoms, *, temperature_K, timestep, tdamp, tchain, tloop):
    n = int(n_atoms)
    kT = units.kB * temperature_K
    Q = np.zeros(tchain)
    Q[0] = 3 * n * kT * tdamp**2
    Q[1:] = kT * tdamp**2
    ndof_kT = 3 * n * kT
    dt2 = timestep / 2
    sub = []
    for coeff in FOURTH_ORDER_COEFFS:
        delta = coeff * dt2 / tloop
        sub.append((delta, delta / 2, -(delta / 4), -delta))
    values = [timestep, dt2, kT, ndof_kT]
    for entry in sub:
        values.extend(entry)
    values.extend(Q.tolist())
    values.extend((1.0 / Q).tolist())
    return np.array(values, dtype=np.float64)


def maxwell_boltzmann_momenta(masses, temperature_K, seed=0):
    masses = np.asarray(masses, dtype=np.float64).reshape(-1)
    rng = seed if isinstance(seed, np.random.Generator) else np.random.default_rng(seed)
    temp = units.kB * temperature_K
    xi = rng.standard_normal((len(masses), 3))
    return xi * np.sqrt(masses * temp)[:, np.newaxis]


class NHC:
    """One system: q, p, F (N, 3) float64, eta/p_eta (M,), E."""

    def __init__(self, masses, positions, momenta, forces, *, temperature_K, timestep, tdamp,
                 tchain=3, tloop=1, f32_kick=False, energy=0.0):
        self.m = np.asarray(masses, dtype=np.float64).reshape(-1, 1)
        self.q = np.array(positions, dtype=np.float64).reshape(-1, 3)
        self.p = np.array(momenta, dtype=np.float64).reshape(-1, 3)
        self.f = np.array(forces, dtype=np.float64).reshape(-1, 3)
        self.M, self.tloop = int(tchain), int(tloop)
        self.eta = np.zeros(self.M)
        self.p_eta = np.zeros(self.M)
        self.E = float(energy)
        self.f32_kick = bool(f32_kick)
        self.c = nhc_constants(self.q.shape[0], temperature_K=temperature_K, timestep=timestep,
                               tdamp=tdamp, tchain=tchain, tloop=tloop)
        self.Q = self.c[C_Q:C_Q + self.M]

    def _ke2(self):
        return float(np.sum(self.p * self.p / self.m))

    def _p_eta_j(self, J, ke2, delta2, neg_delta4):
        pe, Q, M = self.p_eta, self.Q, self.M
        kT, ndof_kT = self.c[2], self.c[3]
        pj = pe[J]
        if J < M - 1:
            s = np.exp(neg_delta4 * pe[J + 1] / Q[J + 1])
            pj = pj * s
        if J == 0:
            g = ke2 - ndof_kT
        else:
            g = pe[J - 1] * pe[J - 1] / Q[J - 1] - kT
        pj = pj + delta2 * g
        if J < M - 1:
            pj = pj * s
        pe[J] = pj

    def _half(self):
        ke2 = self._ke2()
        for _ in range(self.tloop):
            for k in range(3):
                delta, delta2, neg_delta4, neg_delta = self.c[4 + 4 * k: 8 + 4 * k]
                for jj in range(self.M):
                    self._p_eta_j(self.M - 1 - jj, ke2, delta2, neg_delta4)
                for j in range(self.M):
                    self.eta[j] = self.eta[j] + delta * self.p_eta[j] / self.Q[j]
                self.p = self.p * np.exp(neg_delta * self.p_eta[0] / self.Q[0])
                ke2 = self._ke2()
                for j in range(self.M):
                    self._p_eta_j(j, ke2, delta2, neg_delta4)

    def _kick(self, f):
        dt2 = self.c[1]
        if self.f32_kick:
            return (np.float32(dt2) * np.asarray(f, dtype=np.float32)).astype(np.float64)
        return dt2 * np.asarray(f, dtype=np.float64)

    def pre_force(self):
        self._half()
        self.p = self.p + self._kick(self.f)
        self.q = self.q + self.c[0] * self.p / self.m
        return self.q

    def post_force(self, forces, energy=None):
        self.p = self.p + self._kick(forces)
        self._half()
        self.f = np.asarray(forces, dtype=np.float64).reshape(-1, 3).copy()
        if energy is not None:
            self.E = float(energy)

    def flat(self):
        return np.concatenate([self.q.ravel(), self.p.ravel(), self.f.ravel(), self.eta, self.p_eta, [self.E]])

    def kinetic_energy(self):
        return 0.5 * float(np.sum(self.p * (self.p / self.m)))

    def temperature(self):
        return 2 * self.kinetic_energy() / (3 * self.q.shape[0] * units.kB)

    def conserved_energy(self):
        kT, ndof_kT = self.c[2], self.c[3]
        thermostat = ndof_kT * self.eta[0] + kT * self.eta[1:].sum() + (0.5 * self.p_eta**2 / self.Q).sum()
        return self.E + self.kinetic_energy() + thermostat
