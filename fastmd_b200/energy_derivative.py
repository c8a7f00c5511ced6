"""Forces and stress of an energy-tap model by the engine (the surface of fastmd/engine/energy_derivative.py:51,
:87: ``engine_derivative(adapter)`` and ``EnergyDerivative(adapter)(batch, inputs, *, task, n_real)``).

The model exposes ``node_energy(inputs, positions, cell)``: per-atom energies that are differentiable with
respect to the Cartesian positions and the cell (for the MACE-architecture model a
``torch.autograd.Function`` whose backward is the model's explicit edge backward, and whose cell gradient
is its edge virial over the periodic images). One gradient call gives both partial derivatives,
``G_x = dE/dx`` [N, 3] and ``G_L = dE/dL`` [3, 3] (rows of L the lattice vectors), and then

* forces ``F = -G_x``;
* stress (``task`` with ``"s"``), from the response of E to a homogeneous deformation of the whole crystal
  (every position and lattice vector mapped by ``I + e``): ``dE/de = x^T G_x + L^T G_L``, symmetrised
  (only the symmetric part of ``e`` strains the crystal) and divided by the cell volume, in eV/A^3.

The energy is the float64 sum of the first ``n_real`` rows (padding rows follow the real atoms).
"""
from __future__ import annotations

import torch
from torch import Tensor


def cell_volume(cell: Tensor) -> Tensor:
    """|det L| of a [3, 3] cell (rows are lattice vectors)."""
    return torch.linalg.det(cell.to(torch.float64)).abs()


def deformation_derivative(positions: Tensor, grad_positions: Tensor, cell: Tensor, grad_cell: Tensor) -> Tensor:
    """``sym(x^T dE/dx + L^T dE/dL)`` in float64: the derivative of the energy with respect to a symmetric
    homogeneous strain applied to positions and cell together."""
    x, gx = positions.to(torch.float64), grad_positions.to(torch.float64)
    lat, gl = cell.to(torch.float64), grad_cell.to(torch.float64)
    w = x.transpose(0, 1) @ gx + lat.transpose(0, 1) @ gl
    return 0.5 * (w + w.transpose(0, 1))


class EnergyDerivative:
    """The engine's derivative of an energy tap: ``{"e": [1] float64, "f": [forces], "s": [stress]}``."""

    stress_unit = "eV/A^3"

    def __init__(self, adapter) -> None:
        self.adapter = adapter

    def extensive_energy(self, energy: Tensor, atom_counts) -> Tensor:
        """Energy taps return extensive energies already."""
        return energy

    def __call__(self, batch, inputs, *, task: str = "ef", n_real: int | None = None) -> dict:
        want_stress = "s" in task
        positions = batch.positions.detach().requires_grad_(True)
        cell = batch.cell.detach().requires_grad_(want_stress)
        with torch.enable_grad():
            energies = self.adapter.node_energy(inputs, positions, cell)
            count = energies.shape[0] if n_real is None else int(n_real)
            energy = energies[:count].to(torch.float64).sum()
            leaves = [positions, cell] if want_stress else [positions]
            grads = torch.autograd.grad(energy, leaves)
        result = {"e": energy.detach().reshape(1), "f": [-grads[0]]}
        if want_stress:
            virial = deformation_derivative(batch.positions, grads[0], batch.cell, grads[1])
            result["s"] = [(virial / cell_volume(batch.cell)).to(grads[0].dtype)]
        return result


def engine_derivative(adapter) -> EnergyDerivative:
    """The derivative the runtime runs for an adapter with an energy tap (``node_energy``)."""
    if not hasattr(adapter, "node_energy"):
        raise TypeError(f"model adapter {getattr(adapter, 'name', adapter)!r} has no energy tap (node_energy)")
    return EnergyDerivative(adapter)
