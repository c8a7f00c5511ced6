"""Nose-Hoover-chain NVT integrator (ASE 3.29 ``NoseHooverChainNVT``), fp64, on fused sm_100a kernels.

Drop-in for ``fastmd.execution.gpu_nhc.GPUNoseHooverChainNVT`` (gpu_nhc.py:709)
and ``fastmd.execution.replica_batch.ReplicaNoseHooverChainNVT``
(replica_batch.py:314): the same constructor arguments, the
``StatefulIntegrator`` step halves (gpu_integrator.py:69) and observables.

* All state lives in one fp64 device buffer ``[q | p | F | eta | p_eta | E]``
  (R replicas: ``q`` is ``[R*n*3]``, ``eta`` ``[R*M]``, ``E`` ``[R]``), so a
  transactional backup/restore is one copy.
* Each half step is ONE kernel (``fmd_nhc_pre_force`` / ``fmd_nhc_post_force``):
  the whole chain, the kick and the drift, one CTA per replica with the momenta
  in registers; the pre-force half also writes the float32 positions the
  neighbour build and the model read. No host synchronisation, no allocation:
  both halves are CUDA-graph capturable.
* The scalars come from ``nhc_constants`` (the exact Python/NumPy expressions
  of ASE; gpu_nhc.py:113); the kernels are compiled without FMA contraction,
  so every elementwise operation rounds as NumPy's does.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from fastmd_b200 import _lib, units
from fastmd_b200._lib import call, ptr, stream

# Identical Python expressions to ASE's -> identical floats (gpu_nhc.py:90-94)
FOURTH_ORDER_COEFFS = [
    1 / (2 - 2 ** (1 / 3)),
    -(2 ** (1 / 3)) / (2 - 2 ** (1 / 3)),
    1 / (2 - 2 ** (1 / 3)),
]
_C_Q = 16  # index of Q[0] in the device constants (gpu_nhc.py:273-275)
MAX_CHAIN = 8
MAX_ELEMENTS = 32768  # 3n per replica held in one CTA's registers


@dataclass(frozen=True)
class NHCConstants:
    kT: float
    ndof_kT: float
    Q: np.ndarray
    dt2: float
    sub: list
    values: list


def nhc_constants(n_atoms: int, *, temperature_K: float, timestep: float, tdamp: float, tchain: int,
                  tloop: int) -> NHCConstants:
    """ASE's thermostat scalars and the device constants layout (gpu_nhc.py:113):
    dt, dt/2, kT, 3N kT, 3 x (delta, delta/2, -(delta/4), -delta), Q[tchain], 1/Q[tchain]."""
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
    return NHCConstants(kT, ndof_kT, Q, dt2, sub, values)


def maxwell_boltzmann_momenta(masses, temperature_K: float, seed=0) -> np.ndarray:
    """ASE ``MaxwellBoltzmannDistribution(atoms, temperature_K=T, rng=np.random.default_rng(seed))``
    momenta (gpu_nhc.py:199): ``p = xi * sqrt(m kB T)``, ``xi = rng.standard_normal((N, 3))``."""
    masses = np.asarray(masses, dtype=np.float64).reshape(-1)
    rng = seed if isinstance(seed, np.random.Generator) else np.random.default_rng(seed)
    temp = units.kB * temperature_K
    xi = rng.standard_normal((len(masses), 3))
    return xi * np.sqrt(masses * temp)[:, np.newaxis]


class _ChainState:
    """Views into the flat fp64 buffer of R replicas of n atoms, chain length M."""

    def __init__(self, replicas: int, n: int, tchain: int, device) -> None:
        n3 = 3 * n * replicas
        self.flat = torch.zeros(3 * n3 + 2 * replicas * tchain + replicas, dtype=torch.float64, device=device)
        f = self.flat
        self.q = f[0:n3].view(replicas * n, 3)
        self.p = f[n3:2 * n3].view(replicas * n, 3)
        self.f = f[2 * n3:3 * n3].view(replicas * n, 3)
        self.eta = f[3 * n3:3 * n3 + replicas * tchain].view(replicas, tchain)
        self.p_eta = f[3 * n3 + replicas * tchain:3 * n3 + 2 * replicas * tchain].view(replicas, tchain)
        self.energy = f[3 * n3 + 2 * replicas * tchain:]


class _NoseHooverChain:
    """R replicas of one n-atom system, each with its own chain (R = 1: one system)."""

    ensemble = "nvt_nhc"
    comm = None

    def __init__(self, masses, positions, momenta, *, replicas: int, temperature_K: float, timestep: float,
                 tdamp: float, tchain: int = 3, tloop: int = 1, forces=None, potential_energy=None,
                 device="cuda", force_dtype: torch.dtype = torch.float64, numpy_kick_semantics: bool = True) -> None:
        if tchain < 1 or tloop < 1:
            raise ValueError("tchain and tloop must be >= 1")
        if tdamp <= 0 or timestep < 0:
            raise ValueError("tdamp must be positive and timestep non-negative")
        if tchain > MAX_CHAIN:
            raise ValueError(f"tchain <= {MAX_CHAIN} (the chain lives in registers)")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise _lib.FastMDLibraryError("the Nose-Hoover chain kernels run on CUDA devices only")
        masses_np = np.asarray(masses.detach().cpu().numpy() if torch.is_tensor(masses) else masses,
                               dtype=np.float64).reshape(-1)
        self.replicas = int(replicas)
        self.n_atoms = n = int(masses_np.shape[0])
        if 3 * n > MAX_ELEMENTS:
            raise ValueError(f"3n <= {MAX_ELEMENTS} per replica")
        self.tchain, self.tloop = int(tchain), int(tloop)
        self.temperature_K = float(temperature_K)
        self.dt, self.tdamp = float(timestep), float(tdamp)
        self.force_dtype = force_dtype
        self.f32_kick = bool(numpy_kick_semantics and force_dtype == torch.float32)
        c = self._constants(self.temperature_K)
        self._keep(c, self.temperature_K)
        self.consts = torch.tensor(c.values, dtype=torch.float64, device=self.device)
        self.Q = self.consts[_C_Q:_C_Q + self.tchain]
        self.masses = torch.tensor(np.tile(masses_np, self.replicas), dtype=torch.float64,
                                   device=self.device).reshape(-1, 1).contiguous()
        self.state = _ChainState(self.replicas, n, self.tchain, self.device)
        self._backup = _ChainState(self.replicas, n, self.tchain, self.device)
        self.positions32 = torch.zeros(self.replicas * n, 3, dtype=torch.float32, device=self.device)
        self.set_state(positions=positions, momenta=momenta, forces=forces, potential_energy=potential_energy)

    # ---------------------------------------------------------------- constants
    def _constants(self, temperature_K: float) -> NHCConstants:
        return nhc_constants(self.n_atoms, temperature_K=temperature_K, timestep=self.dt, tdamp=self.tdamp,
                             tchain=self.tchain, tloop=self.tloop)

    def _keep(self, c: NHCConstants, temperature_K: float) -> None:
        self.temperature_K = temperature_K
        self.kT, self.ndof_kT, self.Q_np, self.dt2, self.sub = c.kT, c.ndof_kT, c.Q, c.dt2, c.sub

    def set_temperature(self, temperature_K: float) -> None:
        """New target (heating ramp): kT, Q and 3N kT rewritten in place, stream ordered; a
        captured graph reads them at its next replay (gpu_nhc.py:145)."""
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("set_temperature between replays, not inside a capture")
        c = self._constants(float(temperature_K))
        host = torch.tensor(c.values, dtype=torch.float64).pin_memory()
        self.consts.copy_(host, non_blocking=True)
        self._keep(c, float(temperature_K))

    # -------------------------------------------------------------------- state
    @property
    def positions(self) -> Tensor:
        return self.state.q

    @property
    def momenta(self) -> Tensor:
        return self.state.p

    @property
    def forces(self) -> Tensor:
        return self.state.f

    @property
    def eta(self) -> Tensor:
        return self.state.eta

    @property
    def p_eta(self) -> Tensor:
        return self.state.p_eta

    @property
    def potential_energy(self) -> Tensor:
        return self.state.energy

    def _as_f64(self, x) -> Tensor:
        if torch.is_tensor(x):
            return x.detach().to(device=self.device, dtype=torch.float64)
        return torch.as_tensor(np.asarray(x, dtype=np.float64), device=self.device)

    @torch.no_grad()
    def set_state(self, *, positions=None, momenta=None, forces=None, eta=None, p_eta=None,
                  potential_energy=None) -> None:
        """(Re)load state from host or device arrays (not inside a capture)."""
        st = self.state
        for field, value in ((st.q, positions), (st.p, momenta), (st.f, forces)):
            if value is not None:
                field.copy_(self._as_f64(value).reshape(field.shape))
        if positions is not None:
            self.positions32.copy_(st.q)
        for field, value in ((st.eta, eta), (st.p_eta, p_eta), (st.energy, potential_energy)):
            if value is not None:
                field.copy_(self._as_f64(value).reshape(field.shape))

    @torch.no_grad()
    def set_forces(self, forces, energy=None) -> None:
        """F(q) (and E(q)) of the current positions (capture-safe for device tensors)."""
        st = self.state
        st.f.copy_(forces.reshape(st.f.shape) if torch.is_tensor(forces) else self._as_f64(forces).reshape(st.f.shape))
        if energy is not None:
            st.energy.copy_(energy.reshape(st.energy.shape) if torch.is_tensor(energy)
                            else self._as_f64(energy).reshape(st.energy.shape))

    # -------------------------------------------------------------- step halves
    def step_pre_force(self) -> Tensor:
        """ASE ``step()`` first half: NHC(dt/2); p += dt/2 F(q_n); q += dt p / m. Returns the fp64
        positions (updated in place); ``positions32`` holds their float32 copy."""
        call("fmd_nhc_pre_force", ptr(self.state.flat), ptr(self.masses), ptr(self.consts), self.n_atoms,
             self.replicas, self.tchain, self.tloop, int(self.f32_kick), ptr(self.positions32),
             stream(self.device))
        return self.state.q

    def _post_args(self, forces: Tensor, energy: Tensor | None):
        """(float32 forces or None, float64 forces or None, float64 energies or None) for the kernels."""
        forces = forces.reshape(self.replicas * self.n_atoms, 3)
        if not forces.is_contiguous():
            forces = forces.contiguous()
        if forces.dtype == torch.float32:
            f32, f64 = forces, None
        else:
            f32, f64 = None, forces.to(torch.float64)
        e = None
        if energy is not None:
            e = energy.reshape(-1).to(torch.float64)
            if e.numel() != self.replicas:
                raise ValueError(f"energy needs one value per replica ({self.replicas})")
        return f32, f64, e

    def step_post_force(self, forces: Tensor, energy: Tensor | None = None) -> None:
        """ASE ``step()`` second half: p += dt/2 F(q_{n+1}); NHC(dt/2); F (and E) cached.
        ``forces``: ``(R*n, 3)`` float32 or float64 device tensor; ``energy``: R values or None."""
        f32, f64, e = self._post_args(forces, energy)
        call("fmd_nhc_post_force", ptr(self.state.flat), ptr(self.masses), ptr(self.consts), self.n_atoms,
             self.replicas, self.tchain, self.tloop, int(self.f32_kick), ptr(f32), ptr(f64), ptr(e),
             stream(self.device))

    def step_post_pre_force(self, forces: Tensor, energy: Tensor | None = None) -> Tensor:
        """``step_post_force(forces, energy)`` then the next step's ``step_pre_force()`` in one kernel (the
        same state, bitwise): the two halves between two force calls of a whole-step window. Returns the
        fp64 positions of the next step."""
        f32, f64, e = self._post_args(forces, energy)
        call("fmd_nhc_post_pre_force", ptr(self.state.flat), ptr(self.masses), ptr(self.consts), self.n_atoms,
             self.replicas, self.tchain, self.tloop, int(self.f32_kick), ptr(f32), ptr(f64), ptr(e),
             ptr(self.positions32), stream(self.device))
        return self.state.q

    def step(self, force_fn):
        """Full step: ``force_fn(q)`` returns forces or ``(forces, energy)``."""
        q = self.step_pre_force()
        result = force_fn(q)
        forces, energy = result if isinstance(result, tuple) else (result, None)
        self.step_post_force(forces, energy=energy)
        return self.state.q, self.state.p, self.state.f

    # -------------------------------------------------------------- observables
    def _per_replica(self, x: Tensor) -> Tensor:
        return x.reshape(self.replicas, self.n_atoms, 3)

    def velocities(self) -> Tensor:
        return self.state.p / self.masses

    def _kinetic(self) -> Tensor:
        p = self._per_replica(self.state.p)
        m = self.masses.reshape(self.replicas, self.n_atoms, 1)
        return 0.5 * (p * (p / m)).sum(dim=(1, 2))

    def _thermostat(self) -> Tensor:
        st = self.state
        return (self.ndof_kT * st.eta[:, 0] + self.kT * st.eta[:, 1:].sum(dim=1)
                + (0.5 * (st.p_eta * st.p_eta) / self.Q).sum(dim=1))

    def kinetic_energy(self) -> Tensor:
        """0.5 vdot(p, p/m) per replica (fp64)."""
        return self._kinetic()

    def temperature(self) -> Tensor:
        return 2 * self._kinetic() / (3 * self.n_atoms * units.kB)

    def thermostat_energy(self) -> Tensor:
        return self._thermostat()

    def conserved_energy(self, potential_energy=None) -> Tensor:
        epot = self.state.energy if potential_energy is None else potential_energy
        return epot + self._kinetic() + self._thermostat()

    # ------------------------------------------------------------- transactions
    def backup(self) -> None:
        self._backup.flat.copy_(self.state.flat)

    def restore(self) -> None:
        self.state.flat.copy_(self._backup.flat)
        self.positions32.copy_(self.state.q)

    def snapshot(self) -> tuple:
        return self.state.flat.clone(), self._backup.flat.clone()

    def load_snapshot(self, snapshot: tuple) -> None:
        state, backup = snapshot
        self.state.flat.copy_(state)
        self._backup.flat.copy_(backup)
        self.positions32.copy_(self.state.q)


class GPUNoseHooverChainNVT(_NoseHooverChain):
    """One system: ``GPUNoseHooverChainNVT(masses, positions, momenta, temperature_K=, timestep=,
    tdamp=, tchain=3, tloop=1, ...)`` as in gpu_nhc.py:709; observables are 0-dim."""

    def __init__(self, masses, positions, momenta, **kwargs) -> None:
        kwargs.pop("backend", None)  # one backend: the fused kernels
        super().__init__(masses, positions, momenta, replicas=1, **kwargs)

    @classmethod
    def from_atoms(cls, atoms, *, temperature_K, timestep, tdamp, tchain=3, tloop=1, **kwargs):
        return cls(atoms.get_masses(), atoms.get_positions(), atoms.get_momenta(), temperature_K=temperature_K,
                   timestep=timestep, tdamp=tdamp, tchain=tchain, tloop=tloop, **kwargs)

    @property
    def eta(self) -> Tensor:
        return self.state.eta[0]

    @property
    def p_eta(self) -> Tensor:
        return self.state.p_eta[0]

    def kinetic_energy(self) -> Tensor:
        return self._kinetic()[0]

    def temperature(self) -> Tensor:
        return 2 * self._kinetic()[0] / (3 * self.n_atoms * units.kB)

    def thermostat_energy(self) -> Tensor:
        return self._thermostat()[0]

    def conserved_energy(self, potential_energy=None) -> Tensor:
        epot = self.state.energy[0] if potential_energy is None else potential_energy
        return epot + self._kinetic()[0] + self._thermostat()[0]

    def state_dict(self) -> dict:
        return {"eta": self.eta.cpu().numpy().copy(), "p_eta": self.p_eta.cpu().numpy().copy(),
                "temperature_K": self.temperature_K}

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        eta = np.asarray(state["eta"], dtype=np.float64)
        p_eta = np.asarray(state["p_eta"], dtype=np.float64)
        if eta.shape != (self.tchain,) or p_eta.shape != (self.tchain,):
            raise ValueError(f"eta/p_eta must have shape ({self.tchain},)")
        self.set_temperature(float(state["temperature_K"]))
        self.set_state(eta=eta, p_eta=p_eta)


class ReplicaNoseHooverChainNVT(_NoseHooverChain):
    """``replicas`` copies of one system, each with its own chain (replica_batch.py:314):
    ``masses`` ``(n,)``, ``positions``/``momenta`` ``(R, n, 3)`` or ``(R*n, 3)``; observables
    one value per replica."""
