"""Skin-epoch topology reuse for fixed-frame evaluation of one periodic system.

The runner of fastmd/execution/skin_topology.py (``SkinTopologyRunner`` :93) for edges-only models: a
calculator's per-call evaluation (positions in, energy and forces out) that does not rebuild the graph
from scratch. One owner builder keeps the candidate list within ``rc + skin`` (minimum image); every call
re-filters it exactly on the device (``d < rc``) into the padded rows of a capacity bucket, evaluates the
model and reads energy, forces and a status vector back in one synchronisation. With ``capture`` the
re-filter and the model run as one CUDA graph per bucket.

Exactness (skin_topology.py:17-27): the candidate list is the only topology state carried between calls.
The host refreshes it before the launch once an atom moved ``PROACTIVE_REFRESH_FRACTION`` of the skin
since the last refresh (minimum image); the device checks every call that no atom moved half the skin.
A violation, or more pairs than the bucket holds (the padded evaluation is then discarded), redoes the
call after a refresh or in a bucket that fits the exact demand; a truncated candidate row raises
``SkinTopologyUnavailable`` (the caller rebuilds per call). Buckets are selected as the model_graph
runner selects them (``tier`` with ``u_step`` / ``min_pad_u``, the smallest cached bucket above the
demand plus the ``min_pad_u`` margin, skin_topology.py:307). An evaluation equals, bit for bit, the
model's evaluation of a fresh build of the same positions.
"""
from __future__ import annotations


import numpy as np
import torch

from fastmd_b200._capture import quiet_gc

from .graph import FixedCapacityGraphBuilder, fixed_capacity_exceeded
from .model_graph import smallest_fitting_key, tier

# The host refreshes the candidates once an atom moved this fraction of the skin since the last refresh
# (0.9 of the device's limit skin / 2, skin_topology.py:70).
PROACTIVE_REFRESH_FRACTION = 0.45
# Evaluations of one call: the first, a refresh, a growth and one spare (skin_topology.py:86).
_MAX_ATTEMPTS = 4


class SkinTopologyUnavailable(RuntimeError):
    """The skin path cannot evaluate this system (a candidate row is truncated): rebuild per call."""


class SkinTopologyRunner:
    """Fixed-frame energy and forces of one periodic system with a skin-epoch topology
    (skin_topology.py:93). ``model``: an object with ``prepare(batch)`` and
    ``energy_forces_fused(batch, n_systems)`` (``MACEModel``). ``evaluate(positions)`` takes host
    coordinates (float64, any lattice image) and returns ``{"e": float, "f": [n, 3] float32}``.
    ``capture=False`` runs the same body eagerly."""

    def __init__(self, model, *, atomic_numbers, cell, skin: float, capture: bool = True, device="cuda",
                 atom_graph_cutoff: float | None = None, u_step: int = 512, min_pad_u: int = 256, warmup: int = 3,
                 max_neighbors: int | None = None) -> None:
        if not (np.isfinite(skin) and skin > 0):
            raise ValueError("topology reuse needs a positive skin")
        self.model = model
        self.device = torch.device(device)
        self.capture = bool(capture)
        self.skin = float(skin)
        self.u_step, self.min_pad_u, self.warmup = int(u_step), int(min_pad_u), int(warmup)
        self.cell = np.array(cell, dtype=np.float64).reshape(3, 3)
        self._inv_cell = np.linalg.inv(self.cell)
        self.n_real = int(len(atomic_numbers))
        rc = float(atom_graph_cutoff if atom_graph_cutoff is not None else model.config.r_max)
        self.atom_graph_cutoff = rc
        self._builder_args = dict(
            cell=torch.from_numpy(self.cell.astype(np.float32)), atomic_numbers=torch.as_tensor(atomic_numbers),
            atom_graph_cutoff=rc, candidate_cutoff=rc + self.skin, device=self.device, minimum_image=True,
            max_neighbors=max_neighbors)
        # owns the candidate list every bucket's builder reads; its capacity only counts the demand
        self.owner = FixedCapacityGraphBuilder(u_capacity=1, **self._builder_args)
        self.positions = torch.zeros((self.n_real, 3), dtype=torch.float32, device=self.device)
        self._pinned_positions = torch.empty((self.n_real, 3), dtype=torch.float32, pin_memory=True)
        self._pinned_flags = torch.empty(5, dtype=torch.int64, pin_memory=True)
        self._pinned_energy = torch.empty(1, dtype=torch.float64, pin_memory=True)
        self._pinned_forces = torch.empty((self.n_real, 3), dtype=torch.float32, pin_memory=True)
        self.cache: dict[int, dict] = {}
        self.pool = None
        self._reference = None  # host coordinates of the last refresh
        self._demand = None     # undirected pairs of the last evaluation (or refresh)
        self.calls = self.refreshes = self.redo_capacity = self.redo_skin = self.captures = 0
        self.max_host_displacement = 0.0
        self.last_edge_count = 0

    # ------------------------------------------------------------------ buckets
    def _body(self, builder):
        batch, status = builder.build(self.positions, rebuild_candidates=False)
        energy, forces = self.model.energy_forces_fused(batch, n_systems=1)
        flags = torch.cat([status.candidate_valid.reshape(1).long(), status.candidate_capacity_valid.reshape(1).long(),
                           fixed_capacity_exceeded(status, builder).reshape(1).long(), status.edge_count.long(),
                           status.isolated_atom_count.long()])
        return energy, forces, flags

    def _make(self, u_cap: int) -> dict:
        builder = FixedCapacityGraphBuilder(u_capacity=u_cap, candidates_from=self.owner, **self._builder_args)
        self.model.prepare(builder.batch)
        entry = {"builder": builder, "graph": None, "out": None}
        if self.capture:
            side = torch.cuda.Stream(device=self.device)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):  # model buffers and weight splits are made here, not in the capture
                for _ in range(self.warmup):
                    self._body(builder)
            torch.cuda.current_stream().wait_stream(side)
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            graph = torch.cuda.CUDAGraph()
            with quiet_gc(), torch.cuda.graph(graph, pool=self.pool):
                out = self._body(builder)
            entry.update(graph=graph, out=out)
            self.captures += 1
        self.cache[u_cap] = entry
        return entry

    def _bucket(self, u: int) -> dict:
        """The smallest cached bucket strictly above the demand ``u`` (plus the margin), else a new one
        at ``tier``."""
        demand = u + self.min_pad_u
        key = smallest_fitting_key(self.cache.keys(), demand, self.u_step)
        if key is not None:
            return self.cache[key]
        return self._make(tier(demand, self.u_step, self.min_pad_u))

    def close(self) -> None:
        """Release every bucket (graphs and pool)."""
        if self.cache:
            torch.cuda.synchronize(self.device)
        for entry in self.cache.values():
            if entry["graph"] is not None:
                entry["graph"].reset()
        self.cache.clear()
        self.pool = None

    # --------------------------------------------------------------- evaluation
    def _displacement(self, positions: np.ndarray) -> float:
        """The largest distance (A) any atom has moved since the candidates were last built, each atom's
        move taken to its nearest periodic image: fractional moves folded into [-1/2, 1/2)."""
        frac = (positions - self._reference) @ self._inv_cell
        frac -= np.floor(frac + 0.5)
        moved = frac @ self.cell
        return float(np.sqrt((moved * moved).sum(axis=1)).max(initial=0.0))

    def _refresh(self, positions: np.ndarray) -> None:
        """New candidates at the current device positions, then one exact build to learn the pair demand;
        its status comes back in a single host read (truncated candidate rows end the skin reuse)."""
        builder = self.owner
        builder.refresh_candidates(self.positions)
        _, status = builder.build(self.positions, rebuild_candidates=False)
        readout = torch.stack([status.candidate_capacity_valid.reshape(()).to(torch.int64),
                               status.edge_count.reshape(-1)[0].to(torch.int64)]).cpu()
        truncated, n_edges = not bool(readout[0]), int(readout[1])
        if truncated:
            raise SkinTopologyUnavailable(f"candidate rows truncated: more than {builder.buffer_max} candidates "
                                          f"of an atom within {builder.candidate_cutoff} A")
        self._reference = np.array(positions, dtype=np.float64)
        self._demand = -(-n_edges // 2)
        self.refreshes += 1

    def _launch(self, entry):
        if entry["graph"] is not None:
            entry["graph"].replay()
            return entry["out"]
        return self._body(entry["builder"])

    @torch.no_grad()
    def _read(self, energy, forces, flags) -> tuple[list[int], dict]:
        self._pinned_flags.copy_(flags, non_blocking=True)
        self._pinned_energy.copy_(energy.reshape(-1)[:1].to(torch.float64), non_blocking=True)
        self._pinned_forces.copy_(forces[: self.n_real], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._pinned_flags.tolist(), {"e": float(self._pinned_energy[0]),
                                             "f": self._pinned_forces.numpy().copy()}

    @torch.no_grad()
    def evaluate(self, positions) -> dict:
        """Energy (eV, float) and forces ([n, 3] float32, eV/A) of ``positions`` (host, [n, 3])."""
        positions = np.asarray(positions, dtype=np.float64).reshape(self.n_real, 3)
        self._pinned_positions.numpy()[...] = positions
        self.positions.copy_(self._pinned_positions, non_blocking=True)
        if self._reference is None:
            self._refresh(positions)
        else:
            displacement = self._displacement(positions)
            self.max_host_displacement = max(self.max_host_displacement, displacement)
            if displacement >= PROACTIVE_REFRESH_FRACTION * self.skin:
                self._refresh(positions)
        for _ in range(_MAX_ATTEMPTS):
            entry = self._bucket(self._demand)
            flags, result = self._read(*self._launch(entry))
            candidates_valid, capacity_valid, exceeded, edges, _isolated = flags
            if not capacity_valid:
                raise SkinTopologyUnavailable(f"a candidate row exceeds {self.owner.buffer_max} slots")
            if not candidates_valid:
                # an atom moved half the skin without the host test seeing it: refresh, redo
                self.redo_skin += 1
                self._refresh(positions)
                continue
            if exceeded:
                # more pairs than the bucket holds (the padded evaluation is discarded): redo in a bucket
                # that fits this call's exact demand
                self._demand = (edges + 1) // 2
                self.redo_capacity += 1
                continue
            break
        else:
            raise RuntimeError(f"skin topology: no valid evaluation in {_MAX_ATTEMPTS} attempts")
        self._demand = (edges + 1) // 2
        self.last_edge_count = edges
        self.calls += 1
        return result

    def stats(self) -> dict[str, object]:
        return {"calls": self.calls, "refreshes": self.refreshes, "redo_capacity": self.redo_capacity,
                "redo_skin": self.redo_skin, "captures": self.captures, "buckets": sorted(self.cache),
                "max_host_displacement": self.max_host_displacement}


__all__ = ["PROACTIVE_REFRESH_FRACTION", "SkinTopologyRunner", "SkinTopologyUnavailable"]
