"""Engine-owned force/stress derivative of an energy-tap model (fastmd/engine/energy_derivative.py:87).

``EnergyDerivative(adapter)(batch, inputs, task="ef", n_real=None)`` evaluates
``adapter.node_energy(inputs, positions, cell)`` at a fresh position leaf,
sums the real rows in float64 and returns ``{"e": [1] fp64, "f": [forces]}``
(``"s"`` for a task with stress: the strain leaf of the reference,
energy_derivative.py:110-132). The model's ``node_energy`` is a
``torch.autograd.Function`` over libfastmd_b200 kernels, so the derivative is
its explicit backward.
"""
from __future__ import annotations

import torch
from torch import Tensor


def _times(rows: Tensor, matrix: Tensor) -> Tensor:
    """``rows @ matrix`` for a [3, 3] matrix, row by row (no GEMM, no TF32)."""
    return rows[:, 0:1] * matrix[0] + rows[:, 1:2] * matrix[1] + rows[:, 2:3] * matrix[2]


def cell_volume(cell: Tensor) -> Tensor:
    return torch.dot(cell[0], torch.linalg.cross(cell[1], cell[2])).abs()


class EnergyDerivative:
    stress_unit = "eV/A^3"

    def __init__(self, adapter) -> None:
        self.adapter = adapter

    def extensive_energy(self, energy: Tensor, atom_counts) -> Tensor:
        return energy

    def __call__(self, batch, inputs, *, task: str = "ef", n_real: int | None = None) -> dict:
        stress = "s" in task
        with torch.enable_grad():
            leaf = batch.positions.detach().requires_grad_(True)
            positions, cell = leaf, batch.cell
            leaves = (leaf,)
            if stress:  # x' = x (1 + eps), cell' = cell (1 + eps), eps symmetric
                strain = torch.zeros((3, 3), dtype=leaf.dtype, device=leaf.device, requires_grad=True)
                symmetric = 0.5 * (strain + strain.transpose(0, 1))
                positions = leaf + _times(leaf, symmetric)
                cell = cell + _times(cell, symmetric)
                leaves = (leaf, strain)
            energies = self.adapter.node_energy(inputs, positions, cell)
            rows = energies.shape[0] if n_real is None else n_real
            energy = energies[:rows].to(torch.float64).sum()
            grads = torch.autograd.grad(energy, leaves)
        out = {"e": energy.detach().reshape(1), "f": [-grads[0]]}
        if stress:
            out["s"] = [grads[1] / cell_volume(batch.cell)]
        return out


def engine_derivative(adapter) -> EnergyDerivative:
    """The derivative the runtime runs for an energy-tap adapter (energy_derivative.py:51)."""
    if not hasattr(adapter, "node_energy"):
        raise TypeError(f"model adapter {getattr(adapter, 'name', adapter)!r} has no energy tap (node_energy)")
    return EnergyDerivative(adapter)
