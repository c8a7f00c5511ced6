"""Whole-step CUDA-graph MD (fastmd/execution/whole_step_cuda_graph.py:56) and its driver.

``WholeStepGraphRunner`` captures a window of ``steps_per_launch`` MD steps
as ONE CUDA graph: integrator pre-force half -> exact neighbour re-filter ->
model energy and forces -> integrator post-force half, per step, all on
libfastmd_b200 kernels, with the builder's FMD_FLAG_* bits ORed into one
window word. The window is a transaction (whole_step_cuda_graph.py:326-386):
the integrator state is backed up at its start, and ``settle`` reads the
window word once; an invalid window (skin exceeded, candidate or edge
overflow, non-finite state) is rolled back, the candidates are refreshed at
the restored positions, and the window is replayed. A proactive refresh runs
when the last step moved an atom more than ``proactive_refresh_fraction`` of
the skin (whole_step_cuda_graph.py:579-584).

``GPUResidentMolecularDynamics`` (fastmd/interfaces/gpu_md.py:98) wires a
model, a builder and the Nose-Hoover chain together: ``run(steps)``,
``thermodynamics()`` and the host-buffer step ``step_host``, in the
reference's three execution modes (gpu_md.py:104): ``whole_step`` (above),
``model_graph`` (per step: the integrator halves and a ragged neighbour build
eagerly, the model's energy and forces by replay of its capacity bucket's CUDA
graph, fastmd_b200/model_graph.py) and ``eager`` (nothing captured).
"""
from __future__ import annotations


import math

import numpy as np
import torch

from fastmd_b200._capture import quiet_gc
from torch import Tensor

from fastmd_b200.graph import (FLAG_CANDIDATE_OVERFLOW, FLAG_EDGE_OVERFLOW, FLAG_NONFINITE, FLAG_SKIN,
                               FLAG_TRIPLET_OVERFLOW)
_GROW = FLAG_EDGE_OVERFLOW | FLAG_TRIPLET_OVERFLOW  # a capacity the step outgrew: a larger builder
_INVALID = FLAG_SKIN | FLAG_CANDIDATE_OVERFLOW | FLAG_NONFINITE | _GROW
from fastmd_b200.graph import FixedCapacityGraphBuilder, TensorGraphBuilder
from fastmd_b200.gpu_nhc import GPUNoseHooverChainNVT, ReplicaNoseHooverChainNVT, maxwell_boltzmann_momenta
from fastmd_b200.mace import MACEModel, element_index
from fastmd_b200.md_protocol import ExtxyzTrajectory, RestartData
from fastmd_b200.model_graph import BucketedGraphRunner
from fastmd_b200 import units

EXECUTIONS = ("whole_step", "model_graph", "eager")


class FixedCapacityOverflow(RuntimeError):
    """The real graph no longer fits the builder's capacity (whole_step_cuda_graph.py:38)."""


class WholeStepGraphRunner:
    def __init__(self, *, model, builder: FixedCapacityGraphBuilder, integrator, steps_per_launch: int = 1,
                 warmup: int = 3, proactive_refresh_fraction: float = 0.25, fused: bool = True) -> None:
        if steps_per_launch <= 0:
            raise ValueError("steps_per_launch must be positive")
        self.model, self.builder, self.integrator = model, builder, integrator
        # the model evaluation of a step: the fused kernels (default) or the building blocks
        self._evaluate = model.energy_forces_fused if fused else model.energy_forces
        self.steps_per_launch = int(steps_per_launch)
        self.warmup = int(warmup)
        self.proactive_refresh_fraction = float(proactive_refresh_fraction)
        self.replicas = builder.replicas
        self.device = builder.device
        self.window_flags = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.fallbacks = 0
        self.refreshes = 0
        self.eager_steps = 0
        self.capacity_growths = 0
        self.on_resize = None
        self.graph: torch.cuda.CUDAGraph | None = None
        # initial state: candidates at the current positions, F(q0) and E(q0) cached in the integrator
        builder.refresh_candidates(integrator.positions32)
        self.refreshes += 1
        batch, _ = builder.build(integrator.positions32, rebuild_candidates=False)
        self.model.prepare(batch)
        energy, forces = self._evaluate(batch, n_systems=self.replicas)
        integrator.set_forces(forces, energy)
        flags = int(builder.flags.item())
        if flags & FLAG_EDGE_OVERFLOW:
            raise FixedCapacityOverflow(f"{int(batch.n_edges.item())} edges exceed the capacity "
                                        f"{builder.e_capacity}")
        if flags & FLAG_TRIPLET_OVERFLOW:
            raise FixedCapacityOverflow(f"{int(builder.n_triplets.item())} triplets exceed the capacity "
                                        f"{builder.t_capacity}")
        if flags & (FLAG_CANDIDATE_OVERFLOW | FLAG_NONFINITE):
            raise RuntimeError(f"invalid initial graph (flags {flags})")
        self._capture()

    # --------------------------------------------------------------- window
    def _window_body(self) -> None:
        """One window: the pre-force half, then per step the build and the model, and between two steps
        the post-force half and the next pre-force half fused in one launch (``step_post_pre_force``)."""
        integ, builder, model = self.integrator, self.builder, self.model
        integ.backup()
        self.window_flags.copy_(builder.refresh_flags)
        integ.step_pre_force()
        for k in range(self.steps_per_launch):
            batch, _ = builder.build(integ.positions32, rebuild_candidates=False, flags=self.window_flags)
            energy, forces = self._evaluate(batch, n_systems=self.replicas)
            if k + 1 < self.steps_per_launch:
                integ.step_post_pre_force(forces, energy)
            else:
                integ.step_post_force(forces, energy)

    def _capture(self) -> None:
        snapshot = self.integrator.snapshot()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self._window_body()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.integrator.load_snapshot(snapshot)
        graph = torch.cuda.CUDAGraph()
        with quiet_gc(), torch.cuda.graph(graph):
            self._window_body()
        self.integrator.load_snapshot(snapshot)
        self.graph = graph

    def launch(self) -> None:
        """Replay one window (no host synchronisation)."""
        self.graph.replay()

    def settle(self) -> int:
        """Read the window word (one host sync); roll back and redo an invalid window; refresh the
        candidates proactively. Returns the flags of the window as first replayed."""
        flags = int(self.window_flags.item())
        if flags & _INVALID:
            self._fallback(flags)
        elif self.proactive_refresh_fraction > 0:
            moved = float(self.builder.max_displacement.max())
            if moved >= self.proactive_refresh_fraction * self.builder.skin:
                self.builder.refresh_candidates(self.integrator.positions32)
                self.refreshes += 1
        return flags

    def _fallback(self, flags: int) -> None:
        """Roll the window back and redo it (whole_step_cuda_graph.py:477): with more edge capacity
        (a new builder and a recapture) after an overflow; else with candidates refreshed at the
        restored positions; and when even those cannot cover the window, as eager steps that each
        refresh the candidates first. The edges are exact in every route, so the trajectory is the
        same."""
        self.fallbacks += 1
        self.integrator.restore()
        if flags & FLAG_NONFINITE:
            raise FloatingPointError("non-finite positions in the window")
        if flags & _GROW:
            self._grow()
        self.builder.refresh_candidates(self.integrator.positions32)
        self.refreshes += 1
        self.graph.replay()
        again = int(self.window_flags.item())
        if not again & _INVALID:
            return
        self.integrator.restore()
        if again & _GROW:
            self._grow()
            self.builder.refresh_candidates(self.integrator.positions32)
            self.graph.replay()
            if not int(self.window_flags.item()) & _INVALID:
                return
            self.integrator.restore()
        self._eager_window()

    def _eager_window(self) -> None:
        integ, builder, model = self.integrator, self.builder, self.model
        for _ in range(self.steps_per_launch):
            integ.step_pre_force()
            batch, status = builder.build(integ.positions32, rebuild_candidates=True)
            flags = int(status.flags.item())
            if flags & _GROW:
                self._grow()
                batch, status = self.builder.build(integ.positions32, rebuild_candidates=True)
                builder = self.builder
                flags = int(status.flags.item())
            if flags & _INVALID:
                raise RuntimeError(f"invalid graph in an eager step (flags {flags})")
            energy, forces = self._evaluate(batch, n_systems=self.replicas)
            integ.step_post_force(forces, energy)
        self.eager_steps += self.steps_per_launch

    def _grow(self) -> None:
        """Larger capacities and a recapture: the edges (the needed edges + 10 %, pairs rounded to 32) when
        they overflowed, the triplets of a line-graph builder (the needed + 15 %, rounded to 256) when those
        did."""
        old = self.builder
        needed = int(old.batch.n_edges.item())
        u = old.u_capacity
        if needed > old.e_capacity:
            u = int(math.ceil(max(needed * 1.1 / 2, old.u_capacity + 32 * old.replicas) / 32.0)) * 32
        t = None
        if old.n_triplets is not None and int(old.n_triplets.item()) > old.t_capacity:
            wanted = int(old.n_triplets.item())
            t = int(math.ceil(max(wanted * 1.15, old.t_capacity + 256 * old.replicas) / 256.0)) * 256
        self.builder = old.resized(u, t)
        self.graph = None
        self.model.prepare(self.builder.batch)
        self.builder.refresh_candidates(self.integrator.positions32)
        batch, _ = self.builder.build(self.integrator.positions32, rebuild_candidates=False)
        self._evaluate(batch, n_systems=self.replicas)  # buffers of the new size, eagerly
        self.integrator.restore()
        self._capture()
        self.capacity_growths += 1
        if self.on_resize is not None:
            self.on_resize(self.builder)

    def run(self, steps: int) -> None:
        """``steps`` MD steps (a multiple of steps_per_launch), one settle per window."""
        if steps % self.steps_per_launch:
            raise ValueError("steps must be a multiple of steps_per_launch")
        for _ in range(steps // self.steps_per_launch):
            self.launch()
            self.settle()


class GPUResidentMolecularDynamics:
    """NVT Nose-Hoover-chain MD of ``replicas`` copies of one periodic system with the
    MACE-architecture potential (gpu_md.py:98, replica_md.py:224).

    ``positions`` [R*n, 3] (or [n, 3] for one replica), Angstrom; ``momenta`` likewise
    (default Maxwell-Boltzmann at ``temperature_K`` with seed 0 per replica). ``execution``:
    ``"whole_step"`` (windows of ``steps_per_launch`` steps as one CUDA graph), ``"model_graph"``
    or ``"eager"`` (one system; a ragged build per step)."""

    def __init__(self, model, *, positions, cell, atomic_numbers, masses, temperature_K: float,
                 timestep: float, tdamp: float, tchain: int = 3, tloop: int = 1, momenta=None, replicas: int = 1,
                 skin: float = 2.0, u_capacity: int | None = None, steps_per_launch: int = 10,
                 fused: bool = True, execution: str = "whole_step", device="cuda") -> None:
        if execution not in EXECUTIONS:
            raise ValueError(f"execution must be one of {EXECUTIONS}")
        if execution != "whole_step" and int(replicas) != 1:
            raise ValueError(f"execution={execution!r} runs one system; replica ensembles run whole_step")
        self.execution = execution
        self.device = torch.device(device)
        self.replicas = int(replicas)
        n = len(atomic_numbers)
        positions = np.asarray(positions, np.float64).reshape(self.replicas * n, 3)
        if momenta is None:
            momenta = np.concatenate([maxwell_boltzmann_momenta(masses, temperature_K, seed=r)
                                      for r in range(self.replicas)])
        line_model = hasattr(model, "builder_options")  # a model with a bond graph (MatRIS)
        if line_model and execution != "whole_step":
            raise ValueError("a line-graph model (MatRIS) runs execution='whole_step' here")
        cutoff = model.cutoff if line_model else model.config.r_max
        if line_model:
            options = model.builder_options(positions, cell, n, self.replicas)
            if u_capacity is not None:
                options["u_capacity"] = u_capacity
        else:
            if u_capacity is None:
                # MACE's capacity tiers (mace.py:70, CapacityStep(32, 32, 1.02)) from the initial pair count
                pairs = self._initial_pairs(positions[:n], cell, cutoff)
                u_capacity = int(math.ceil(max(pairs * 1.08, pairs + 32) / 32.0)) * 32 * self.replicas
            options = dict(u_capacity=u_capacity)
        self.builder = FixedCapacityGraphBuilder(
            cell=torch.as_tensor(np.asarray(cell), dtype=torch.float32), atomic_numbers=torch.as_tensor(atomic_numbers),
            atom_graph_cutoff=cutoff, candidate_cutoff=cutoff + skin, device=self.device, replicas=self.replicas,
            **options)
        kw = dict(temperature_K=temperature_K, timestep=timestep, tdamp=tdamp, tchain=tchain, tloop=tloop,
                  force_dtype=torch.float32, device=self.device)
        if self.replicas == 1:
            self.integrator = GPUNoseHooverChainNVT(masses, positions, momenta, **kw)
        else:
            self.integrator = ReplicaNoseHooverChainNVT(masses, positions, momenta, replicas=self.replicas, **kw)
        self.model = model
        self.n_atoms = n
        self.steps_done = 0
        self.numbers = np.asarray(atomic_numbers, np.int64).reshape(-1)
        self.cell = np.asarray(cell, np.float64).reshape(3, 3)
        if execution == "whole_step":
            self.runner = WholeStepGraphRunner(model=model, builder=self.builder, integrator=self.integrator,
                                               steps_per_launch=steps_per_launch, fused=fused)
            self.runner.on_resize = self._resized
            return
        # model_graph / eager: a ragged build per step (gpu_graph_builder.py:935), F(q0) first
        self.ragged = TensorGraphBuilder(cell=torch.as_tensor(np.asarray(cell), dtype=torch.float32),
                                         atomic_numbers=torch.as_tensor(atomic_numbers), atom_graph_cutoff=cutoff,
                                         device=self.device)
        self._element = None
        self.runner = BucketedGraphRunner(model) if execution == "model_graph" else None
        energy, forces = self._evaluate(self.ragged.build(self.integrator.positions32))
        self.integrator.set_forces(forces, energy)

    def _evaluate(self, batch):
        """Energies and forces of a ragged build: replay of its bucket, or the fused kernels eagerly."""
        if self.runner is not None:
            return self.runner.run(batch)
        if self._element is None:  # element rows once (a host conversion), reused every step
            self.model.prepare(batch)
            self._element = (batch.element, batch.element64)
        batch.element, batch.element64 = self._element
        return self.model.energy_forces_fused(batch)

    def _step(self) -> None:
        integ = self.integrator
        integ.step_pre_force()
        energy, forces = self._evaluate(self.ragged.build(integ.positions32))
        integ.step_post_force(forces, energy)

    def _resized(self, builder) -> None:
        self.builder = builder

    @staticmethod
    def _initial_pairs(positions, cell, cutoff) -> int:
        from fastmd_b200.graph import neighbor_list

        pos = torch.as_tensor(positions, dtype=torch.float32).cuda()
        center, _, _, _ = neighbor_list(pos, torch.as_tensor(np.asarray(cell), dtype=torch.float32), cutoff)
        return int(center.shape[0] + 1) // 2

    def run(self, steps: int) -> None:
        if self.execution == "whole_step":
            self.runner.run(steps)
        else:
            for _ in range(steps):
                self._step()
        self.steps_done += steps

    # ------------------------------------------------------------ restart files and frames
    def restart_data(self, parameters: dict | None = None, offsets: dict | None = None) -> RestartData:
        """The current state as a restart file's contents (md_protocol.py:123): one system, rows in ID
        order, the cached forces and energy of the state, the chain, ``engine`` "native"."""
        if self.replicas != 1:
            raise ValueError("a restart file holds one system")
        integ = self.integrator
        weights = getattr(self.model, "weights_host", None)  # MACE's per-element reference energies; MatRIS has none
        e0 = (np.asarray(weights["e0"], np.float64)[element_index(self.numbers)] if weights is not None
              else np.zeros(self.n_atoms))
        params = {"ensemble": "nvt_nhc", "tchain": integ.tchain, "tloop": integ.tloop, "timestep": integ.dt,
                  "tdamp": integ.tdamp, "execution": self.execution, **(parameters or {})}
        return RestartData(
            ids=np.arange(self.n_atoms, dtype=np.int64), numbers=self.numbers.copy(),
            masses=integ.masses.cpu().numpy().astype(np.float64), positions=integ.state.q.cpu().numpy().copy(),
            momenta=integ.state.p.cpu().numpy().copy(), forces=integ.state.f.cpu().numpy().astype(np.float32),
            energy=integ.state.energy.cpu().numpy().copy(), reference_energy=np.array([e0.sum()]),
            cell=self.cell.copy(), pbc=np.ones(3, bool), step=int(self.steps_done), parameters=params,
            temperature_K=float(integ.temperature_K), nhc_state=integ.state_dict(), offsets=dict(offsets or {}),
            engine="native")

    def load_restart(self, data: RestartData) -> None:
        """Continue from a restart file's state: positions, momenta, the cached forces and energy (not
        re-evaluated), the chain and the step count; the candidates are rebuilt at the positions."""
        if self.replicas != 1 or len(data.numbers) != self.n_atoms or not np.array_equal(
                np.asarray(data.numbers)[np.argsort(data.ids)], self.numbers):
            raise ValueError("the restart file holds another system")
        order = np.argsort(np.asarray(data.ids))
        integ = self.integrator
        integ.set_state(positions=np.asarray(data.positions, np.float64)[order],
                        momenta=np.asarray(data.momenta, np.float64)[order],
                        forces=np.asarray(data.forces, np.float64)[order],
                        potential_energy=np.asarray(data.energy, np.float64).reshape(-1))
        if data.nhc_state is not None:
            integ.load_state_dict(data.nhc_state)
        self.steps_done = int(data.step)
        if self.execution == "whole_step":
            self.builder.refresh_candidates(integ.positions32)

    def write_frame(self, trajectory: ExtxyzTrajectory, info: dict | None = None) -> None:
        """The current state as one extxyz frame (velocities = momenta / masses, the cached forces)."""
        if self.replicas != 1:
            raise ValueError("a frame holds one system")
        integ = self.integrator
        p, m = integ.state.p.cpu().numpy(), integ.masses.cpu().numpy()
        trajectory.write(numbers=self.numbers, positions=integ.state.q.cpu().numpy(), cell=self.cell,
                         pbc=np.ones(3, bool), velocities=p / m[:, None], forces=integ.state.f.cpu().numpy(),
                         energy=float(integ.state.energy[0]), info={"step": self.steps_done, **(info or {})})

    def thermodynamics(self) -> dict:
        """Per-replica potential, kinetic and conserved energy (eV) and temperature (K)."""
        integ = self.integrator
        return {"potential_energy": integ.state.energy.cpu().numpy().copy(),
                "kinetic_energy": np.atleast_1d(integ.kinetic_energy().cpu().numpy()).copy(),
                "temperature": np.atleast_1d(integ.temperature().cpu().numpy()).copy(),
                "conserved_energy": np.atleast_1d(integ.conserved_energy().cpu().numpy()).copy()}

    def step_host(self, positions: Tensor, momenta: Tensor, out: dict) -> None:
        """One window from HOST state: upload positions and momenta (pinned), replay, settle, and
        download positions, momenta, forces and energies into the pinned ``out`` buffers."""
        if self.execution != "whole_step":
            raise RuntimeError("step_host replays whole-step windows (execution='whole_step')")
        integ = self.integrator
        integ.state.q.copy_(positions, non_blocking=True)
        integ.state.p.copy_(momenta, non_blocking=True)
        integ.positions32.copy_(integ.state.q)
        self.runner.launch()
        self.runner.settle()
        out["positions"].copy_(integ.state.q, non_blocking=True)
        out["momenta"].copy_(integ.state.p, non_blocking=True)
        out["forces"].copy_(integ.state.f, non_blocking=True)
        out["energy"].copy_(integ.state.energy, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
