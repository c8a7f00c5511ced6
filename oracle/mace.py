"""FP64 CPU restatement of the MACE-architecture potential -- test oracle (parity unpinned).

The reference evaluates MACE through upstream mace-torch 0.3.16 +
cuEquivariance 0.9.1 (pyproject.toml:20, :26; call sites fastmd/models/mace.py:143-156,
:356-388), neither of which is part of the reference tree nor installed here,
and the reference's own MACE tests compare against mace-torch itself with no
stored values (tests/adapters/test_mace_adapter.py:320-540). This oracle is a
restatement of the published MACE equations (Batatia et al., NeurIPS 2022)
at l <= 1, correlation 3, in float64 torch on the CPU with autograd forces;
the product's kernels are checked against it, not against mace-torch:
**parity unpinned** for this model.

Pinned pieces it shares with the reference: the radial basis
``sqrt(2/rc) sin(n pi d/rc)/d * envelope(d/rc)`` is the reference's
``BesselExpansion`` + ``PolynomialEnvelope`` (fastmd/models/matris/basis_function.py:139, :31),
checked against golden vectors of that module; the edge vectors follow the
MACE adapter's convention (mace.py:363-385: the engine's centre <- neighbour
edge with its integer image).
"""
from __future__ import annotations

import math

import numpy as np
import torch


def bessel_envelope(d, r_max, n_basis, p):
    """[E, n_basis] radial features (basis_function.py:185 with the envelope of :31)."""
    n = torch.arange(1, n_basis + 1, dtype=d.dtype)
    x = d / r_max
    a, b, c = -(p + 1) * (p + 2) / 2, p * (p + 2), -p * (p + 1) / 2
    env = 1 + a * x**p + b * x ** (p + 1) + c * x ** (p + 2)
    env = torch.where(x < 1, env, torch.zeros_like(env))
    return math.sqrt(2.0 / r_max) * torch.sin(n * math.pi * d[:, None] / r_max) / d[:, None] * env[:, None]


def silu(x):
    return x * torch.sigmoid(x)


def energy_forces(weights: dict, config, positions, cell, atomic_numbers, edges, images, *, n_systems=1,
                  dtype=torch.float64, stress=False):
    """(per-system energies [R], forces [N, 3], node energies [N]) in float64, and the stress [3, 3]
    (eV/A^3) after them with ``stress``.

    ``edges`` [E, 2] (centre i, neighbour j), ``images`` [E, 3] integer images: the edge vector
    is x_j + image @ cell - x_i, messages flow j -> i. The stress is the reference's strain leaf
    (fastmd/engine/energy_derivative.py:110-132): x' = x + x eps, cell' = cell + cell eps with a
    symmetric eps, s = dE/d(eps) / |det cell|."""
    W = {k: torch.as_tensor(np.asarray(v), dtype=dtype if v.dtype != np.float64 else torch.float64)
         for k, v in weights.items()}
    C = config.channels
    pos = torch.as_tensor(np.asarray(positions, np.float64), dtype=dtype).clone().requires_grad_(True)
    cell = torch.as_tensor(np.asarray(cell, np.float64), dtype=dtype).reshape(3, 3)
    z = torch.as_tensor(np.asarray(atomic_numbers, np.int64)) - 1
    edges = torch.as_tensor(np.asarray(edges, np.int64))
    images = torch.as_tensor(np.asarray(images, np.float64), dtype=dtype)
    N = pos.shape[0]
    i, j = edges[:, 0], edges[:, 1]
    strain = torch.zeros(3, 3, dtype=dtype, requires_grad=True)
    sym = 0.5 * (strain + strain.T)
    pos_s, cell_s = (pos + pos @ sym, cell + cell @ sym) if stress else (pos, cell)
    r = pos_s[j] + images @ cell_s - pos_s[i]
    d = torch.linalg.vector_norm(r, dim=1)
    Y = math.sqrt(3.0) * r / d[:, None]
    phi = bessel_envelope(d, config.r_max, config.num_bessel, config.poly_p)
    s = W["embedding"][z]
    v = None
    terms = []
    for L in range(config.num_interactions):
        last = L == config.num_interactions - 1
        P = config.paths(L)
        p = f"{L}."
        h = silu(phi @ W[p + "radial.0"].T)
        h = silu(h @ W[p + "radial.1"].T)
        h = silu(h @ W[p + "radial.2"].T)
        R = (h @ W[p + "radial.3"].T).reshape(-1, P, C)
        s_t = s @ W[p + "up0"].T
        m0 = R[:, 0] * s_t[j]
        m1 = (R[:, 1] * s_t[j])[:, None, :] * Y[:, :, None]
        if P == 4:
            v_t = torch.einsum("nxc,dc->nxd", v, W[p + "up1"])
            vj = v_t[j]
            m1 = m1 + R[:, 2][:, None, :] * vj
            m0 = m0 + R[:, 3] * torch.einsum("exc,ex->ec", vj, Y) / math.sqrt(3.0)
        A0 = torch.zeros(N, C, dtype=dtype).index_add(0, i, m0) / config.avg_num_neighbors
        A1 = torch.zeros(N, 3, C, dtype=dtype).index_add(0, i, m1) / config.avg_num_neighbors
        A0 = A0 @ W[p + "lin0"].T
        A1 = torch.einsum("nxc,dc->nxd", A1, W[p + "lin1"])
        q = (A1 * A1).sum(dim=1)
        w0 = W[p + "prod0"][z]
        B0 = w0[:, 0] * A0 + w0[:, 1] * A0**2 + w0[:, 2] * q + w0[:, 3] * A0**3 + w0[:, 4] * A0 * q
        s_new = B0 @ W[p + "out0"].T
        if L > 0:
            s_new = s_new + torch.einsum("nc,ncd->nd", s, W[p + "skip0"][z])
        v_new = None
        if not last:
            u = W[p + "prod1"][z]
            c = u[:, 0] + u[:, 1] * A0 + u[:, 2] * A0**2 + u[:, 3] * q
            B1 = c[:, None, :] * A1
            v_new = torch.einsum("nxc,dc->nxd", B1, W[p + "out1"])
            if L > 0 and v is not None:
                v_new = v_new + torch.einsum("nxc,ncd->nxd", v, W[p + "skip1"][z])
        if L == 0:
            terms.append((s_new @ W["readout.0"].T)[:, 0])
        if last:
            terms.append((silu(s_new @ W["readout.1a"].T) @ W["readout.1b"].T)[:, 0])
        s, v = s_new, v_new
    e0 = torch.as_tensor(np.asarray(weights["e0"], np.float64))
    node = e0[z] + config.scale * sum(t.to(torch.float64) for t in terms) + config.shift
    totals = node.reshape(n_systems, -1).sum(dim=1)
    if not stress:
        (grad,) = torch.autograd.grad(totals.sum(), pos)
        return totals.detach().numpy(), (-grad).detach().numpy(), node.detach().numpy()
    grad, gstrain = torch.autograd.grad(totals.sum(), (pos, strain))
    volume = abs(float(torch.linalg.det(cell)))
    return (totals.detach().numpy(), (-grad).detach().numpy(), node.detach().numpy(),
            (gstrain / volume).detach().numpy())
