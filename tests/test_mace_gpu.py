"""The MACE-architecture potential on the GPU kernels against the FP64 oracle (parity unpinned for
the model itself: its oracle restates the published equations; the radial basis is pinned to the
reference's BesselExpansion)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import mace as omace
from oracle import neighbors as onb

pytestmark = pytest.mark.gpu

# the tolerance of the benchmark contract: per-step energies and forces within 1e-5 relative (fp32)
REL = 1e-5


def _system(seed=0):
    from fastmd_b200.structures import perovskite

    return perovskite(seed=seed)


def _graph(pos, cell, numbers, cuda, replicas=1, u_capacity=4096):
    from fastmd_b200.graph import FixedCapacityGraphBuilder

    b = FixedCapacityGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32), atomic_numbers=torch.tensor(numbers),
                                  u_capacity=u_capacity * replicas, atom_graph_cutoff=6.0, candidate_cutoff=8.0,
                                  device=cuda, replicas=replicas)
    batch, status = b.build(torch.from_numpy(np.asarray(pos, np.float32)).to(cuda))
    assert int(status.flags.item()) == 0
    return b, batch


def _oracle(model, batch, numbers, replicas=1):
    n = int(batch.n_edges.item())
    edges = batch.edge_index[:n].cpu().numpy()
    images = batch.edge_image[:n].cpu().numpy().round()
    return omace.energy_forces(model.weights_host, model.config, batch.positions.cpu().numpy().astype(np.float64),
                               batch.cell.cpu().numpy(), np.tile(numbers, replicas), edges, images,
                               n_systems=replicas)


@pytest.mark.parametrize("tag", ["mace", "matris"])
def test_radial_basis_kernel_matches_reference_module(cuda, tag):
    from fastmd_b200._lib import call, ptr, stream

    g = golden("radial")
    n, rc, p = g[f"radial_{tag}_params"]
    d = g["radial_d"]
    E = d.size
    pos = np.zeros((E + 1, 3), np.float32)
    pos[1:, 0] = d
    edge_index = np.stack([np.zeros(E), np.arange(1, E + 1)], 1).astype(np.int32)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)  # noqa: E731
    # every device buffer stays referenced until the kernel has run
    cell, pos_t, edges_t, images_t = (t(np.eye(3, dtype=np.float32) * 50.0), t(pos), t(edge_index),
                                      t(np.zeros((E, 3), np.float32)))
    ysh = torch.empty(E, 4, device=cuda)
    phi = torch.empty(E, int(n), device=cuda)
    call("fmd_mace_edge_geometry", ptr(pos_t), ptr(cell), ptr(edges_t), ptr(images_t), E, float(rc), int(n), int(p),
         ptr(ysh), ptr(phi), stream(cuda))
    torch.cuda.synchronize()
    np.testing.assert_allclose(phi.cpu().numpy(), g[f"radial_{tag}"], rtol=2e-5, atol=2e-6)
    assert torch.equal(ysh[:, 3].cpu(), torch.from_numpy(d))


def _close(mine, ref, rel=REL):
    scale = max(float(np.abs(ref).max()), 1e-12)
    err = float(np.abs(np.asarray(mine, np.float64) - ref).max())
    assert err <= rel * scale, (err, scale)


def test_energy_forces_match_fp64_oracle(cuda):
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers, _ = _system(0)
    model = MACEModel(device=cuda)
    _, batch = _graph(pos, cell, numbers, cuda)
    energy, forces = model.energy_forces(batch)
    E, F, node = _oracle(model, batch, numbers)
    _close(energy.cpu().numpy(), E, 1e-7)
    _close(model.buffers(batch.positions.shape[0], batch.edge_index.shape[0]).t["node_energy"].cpu().numpy(), node,
           1e-6)
    _close(forces.cpu().numpy(), F)
    assert float(np.abs(F).max()) > 0.05  # the forces are not trivially small


def test_energy_derivative_autograd_route_equals_explicit_backward(cuda):
    from fastmd_b200.energy_derivative import EnergyDerivative
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers, _ = _system(1)
    model = MACEModel(device=cuda)
    _, batch = _graph(pos, cell, numbers, cuda)
    energy, forces = model.energy_forces(batch)
    energy, forces = energy.clone(), forces.clone()
    out = EnergyDerivative(model)(batch, batch, task="ef", n_real=batch.positions.shape[0])
    assert torch.equal(out["e"], energy)
    assert torch.equal(out["f"][0], forces)


def test_stress_matches_fp64_oracle(cuda):
    """EnergyDerivative(task="efs"): the deformation derivative from the position and cell gradients
    (fmd_mace_edge_virial) against the FP64 oracle's own strain leaf."""
    from fastmd_b200.energy_derivative import EnergyDerivative
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers, _ = _system(2)
    model = MACEModel(device=cuda)
    _, batch = _graph(pos, cell, numbers, cuda)
    out = EnergyDerivative(model)(batch, batch, task="efs", n_real=batch.positions.shape[0])
    n = int(batch.n_edges.item())
    E, F, _, S = omace.energy_forces(model.weights_host, model.config, batch.positions.cpu().numpy().astype(np.float64),
                                     batch.cell.cpu().numpy(), numbers, batch.edge_index[:n].cpu().numpy(),
                                     batch.edge_image[:n].cpu().numpy().round(), stress=True)
    _close(out["e"].cpu().numpy(), E, 1e-7)
    _close(out["f"][0].cpu().numpy(), F)
    s = out["s"][0].cpu().numpy()
    assert s.shape == (3, 3) and np.allclose(s, s.T, atol=1e-6 * np.abs(S).max())
    _close(s, S, 1e-4)
    assert float(np.abs(S).max()) > 1e-4  # not trivially zero


def test_small_channel_model_matches_oracle_and_is_deterministic(cuda):
    from fastmd_b200.mace import MACEConfig, MACEModel

    pos, cell, numbers, _ = _system(2)
    model = MACEModel(MACEConfig(channels=32, num_interactions=3), device=cuda, seed=3)
    _, batch = _graph(pos, cell, numbers, cuda)
    e1, f1 = (x.clone() for x in model.energy_forces(batch))
    e2, f2 = model.energy_forces(batch)
    assert torch.equal(e1, e2) and torch.equal(f1, f2)
    E, F, _ = _oracle(model, batch, numbers)
    _close(e1.cpu().numpy(), E, 1e-7)
    _close(f1.cpu().numpy(), F)


def test_replica_union_energies_equal_single_systems(cuda):
    from fastmd_b200.mace import MACEModel

    R = 3
    systems = [_system(seed) for seed in range(R)]
    cell, numbers = systems[0][1], systems[0][2]
    model = MACEModel(device=cuda)
    _, batch = _graph(np.concatenate([s[0] for s in systems]), cell, numbers, cuda, replicas=R)
    energy, forces = model.energy_forces(batch, n_systems=R)
    energy, forces = energy.clone(), forces.clone()
    N = numbers.size
    for r, s in enumerate(systems):
        _, single = _graph(s[0], cell, numbers, cuda)
        e, f = model.energy_forces(single)
        assert torch.equal(energy[r:r + 1], e)
        assert torch.equal(forces[r * N:(r + 1) * N], f)


def test_forces_sum_to_zero_and_translation_invariance(cuda):
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers, _ = _system(4)
    model = MACEModel(device=cuda)
    _, batch = _graph(pos, cell, numbers, cuda)
    e0, f0 = (x.clone() for x in model.energy_forces(batch))
    assert float(f0.double().sum(0).abs().max()) < 1e-4
    _, moved = _graph(pos + np.array([0.37, -1.1, 2.3]), cell, numbers, cuda)
    e1, f1 = model.energy_forces(moved)
    assert abs(float(e1 - e0)) < 1e-9 * abs(float(e0)) + 2e-4
    _close(f1.cpu().numpy(), f0.cpu().numpy().astype(np.float64), 1e-4)


@pytest.mark.parametrize("channels,layers,seed", [(128, 2, 0), (32, 3, 2), (64, 1, 3)])
def test_fused_step_matches_fp64_oracle(cuda, channels, layers, seed):
    from fastmd_b200.mace import MACEConfig, MACEModel

    pos, cell, numbers, _ = _system(seed)
    model = MACEModel(MACEConfig(channels=channels, num_interactions=layers), device=cuda, seed=seed + 1)
    _, batch = _graph(pos, cell, numbers, cuda)
    energy, forces = model.energy_forces_fused(batch)
    E, F, _ = _oracle(model, batch, numbers)
    _close(energy.cpu().numpy(), E, 1e-7)
    _close(forces.cpu().numpy(), F)
    e2, f2 = model.energy_forces_fused(batch)
    assert torch.equal(e2, energy) and torch.equal(f2, forces)  # deterministic
    eu, fu = model.energy_forces(batch)
    _close(fu.cpu().numpy(), forces.cpu().numpy().astype(np.float64))


@pytest.mark.parametrize("R", [3, 5])
def test_fused_replica_union_equals_single_systems(cuda, R):
    """R = 5: the union's 175 atom groups run 4 atoms per CTA, a single system's 35 one atom per CTA
    (fewer groups than SMs); on the SIMT edge kernels the results do not depend on the grouping (the
    default precision moves a union of 8,192 edge rows or more to the tensor-core radial path, whose
    results match within the FP32 bar instead)."""
    from fastmd_b200.mace import MACEModel

    systems = [_system(seed) for seed in range(R)]
    cell, numbers = systems[0][1], systems[0][2]
    model = MACEModel(device=cuda, radial_precision="ieee")
    _, batch = _graph(np.concatenate([s[0] for s in systems]), cell, numbers, cuda, replicas=R)
    energy, forces = (x.clone() for x in model.energy_forces_fused(batch, n_systems=R))
    N = numbers.size
    for r, s in enumerate(systems):
        _, single = _graph(s[0], cell, numbers, cuda)
        e, f = model.energy_forces_fused(single)
        assert torch.equal(energy[r:r + 1], e)
        assert torch.equal(forces[r * N:(r + 1) * N], f)


def test_fused_tensor_core_radial_matches_oracle(cuda):
    """The radial MLPs and their backward as the tcgen05 3xTF32 GEMM chain, and the node kernels' channel
    mixings as grouped tcgen05 GEMMs (forced on the 135-atom graph), against the FP64 oracle and the IEEE
    CUDA-core kernels, to the benchmark's 1e-5."""
    from fastmd_b200.mace import MACEModel
    from fastmd_b200.ops import read_flags

    pos, cell, numbers, _ = _system(0)
    _, batch = _graph(pos, cell, numbers, cuda)
    read_flags(cuda)
    tc = MACEModel(device=cuda, radial_precision="tf32x3")
    energy, forces = (x.clone() for x in tc.energy_forces_fused(batch))
    assert next(iter(tc._fused_bufs.values())).tensor_core_radial
    assert next(iter(tc._fused_bufs.values())).tensor_core_nodes
    E, F, _ = _oracle(tc, batch, numbers)
    _close(energy.cpu().numpy(), E)
    _close(forces.cpu().numpy(), F)
    ieee = MACEModel(device=cuda, radial_precision="ieee")
    ei, fi = ieee.energy_forces_fused(batch)
    assert not next(iter(ieee._fused_bufs.values())).tensor_core_radial
    _close(forces.cpu().numpy(), fi.cpu().numpy().astype(np.float64))
    e2, f2 = tc.energy_forces_fused(batch)
    assert torch.equal(e2, energy) and torch.equal(f2, forces)  # deterministic
    assert read_flags(cuda) == 0


def test_fused_tensor_core_radial_on_a_large_union(cuda):
    """32 replicas (about 70k edge rows, above the 8,192-row threshold): the default precision takes
    the tensor-core radial path; per-replica energies and forces match the IEEE path and, for replica 0,
    the FP64 oracle of the single system."""
    from fastmd_b200.mace import MACEModel

    R = 32
    systems = [_system(seed) for seed in range(R)]
    cell, numbers = systems[0][1], systems[0][2]
    N = numbers.size
    _, batch = _graph(np.concatenate([s[0] for s in systems]), cell, numbers, cuda, replicas=R, u_capacity=1100)
    assert batch.edge_index.shape[0] >= 65536
    auto = MACEModel(device=cuda)
    energy, forces = (x.clone() for x in auto.energy_forces_fused(batch, n_systems=R))
    assert next(iter(auto._fused_bufs.values())).tensor_core_radial
    assert next(iter(auto._fused_bufs.values())).tensor_core_nodes
    ieee = MACEModel(device=cuda, radial_precision="ieee")
    ei, fi = ieee.energy_forces_fused(batch, n_systems=R)
    for r in range(R):
        _close(energy[r].cpu().numpy(), ei[r].cpu().numpy())
        _close(forces[r * N:(r + 1) * N].cpu().numpy(), fi[r * N:(r + 1) * N].cpu().numpy().astype(np.float64))
    _, single = _graph(systems[0][0], cell, numbers, cuda)
    E, F, _ = _oracle(auto, single, numbers)
    _close(energy[0].cpu().numpy(), E)
    _close(forces[:N].cpu().numpy(), F)
