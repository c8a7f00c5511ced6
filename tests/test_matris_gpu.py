"""The MatRIS-10M potential on the GPU (fastmd_b200.matris) against the reference's own model.

Energies, forces and stress of the config-0 perovskite with the seeded weights, (a) on the reference's
legacy CPU graph from the fixture and (b) on this build's fixed-capacity graph (sink padding, capacity
rows), against the FP64 truth (the oracle, pinned to the reference's float64 evaluation to 1e-10) and
against the reference's float32 evaluation. Bounds: energy 1e-6 relative; stress 1e-5 of its largest
component; forces within twice the reference's own float32 error (at least 1e-5 of the largest force):
the reference's float32 forces sit 2.6e-5 to 3.1e-5 of the largest force from the FP64 result.
"""
import numpy as np
import pytest
import torch

from conftest import golden
from fastmd_b200.matris_params import MATRIS_10M, seeded_parameters
from oracle import matris as om

pytestmark = pytest.mark.gpu

_TRUTH = {}


def _truth(g, seed):
    """FP64 oracle result at the float32 coordinates the float32 evaluations see."""
    if seed not in _TRUTH:
        t = f"matris_s{seed}"
        _TRUTH[seed] = om.energy_forces_stress(
            seeded_parameters(MATRIS_10M, 0), MATRIS_10M, g[f"{t}_positions"].astype(np.float64), g[f"{t}_cell"],
            g[f"{t}_numbers"], g[f"{t}_edge_index"], g[f"{t}_edge_image"], g[f"{t}_d2u"], g[f"{t}_u2d"],
            g[f"{t}_line_graph"])
    return _TRUTH[seed]


def _check(g, seed, energy, forces, stress, e_tol=1e-5):
    t = f"matris_s{seed}"
    e_ref, f_ref, s_ref = _truth(g, seed)
    ref32_err = np.abs(g[f"{t}_f32"] - f_ref).max()
    fmax = np.abs(f_ref).max()
    e, f, s = float(energy[0]), forces.cpu().numpy().astype(np.float64), stress.cpu().numpy().astype(np.float64)
    assert abs(e - e_ref) <= e_tol * abs(e_ref), (e, e_ref)
    assert np.abs(f - f_ref).max() <= max(2.0 * ref32_err, 1e-5 * fmax), (np.abs(f - f_ref).max(), ref32_err, fmax)
    assert np.abs(s - s_ref).max() <= 1e-5 * np.abs(s_ref).max(), (s, s_ref)
    # and against the reference's own float32 evaluation
    assert abs(e - float(g[f"{t}_e32"])) <= e_tol * abs(e_ref)
    assert np.abs(f - g[f"{t}_f32"]).max() <= 3.0 * ref32_err


_MODELS = {}


def _model(cuda, precision="tf32x3"):
    from fastmd_b200.matris import MatRISModel

    if precision not in _MODELS:
        _MODELS[precision] = MatRISModel(MATRIS_10M, seed=0, device=cuda, precision=precision)
    return _MODELS[precision]


@pytest.fixture(scope="module")
def model(cuda):
    return _model(cuda)


# energy bounds: the north-star 1e-5 with the 3xTF32 tensor-core GEMMs, 1e-6 on the IEEE FP32 path
@pytest.mark.parametrize("precision,e_tol", [("tf32x3", 1e-5), ("ieee", 1e-6)])
@pytest.mark.parametrize("seed", [0, 1])
def test_matris_on_the_reference_graph(cuda, seed, precision, e_tol):
    from fastmd_b200.matris import MatRISGraph

    model = _model(cuda, precision)
    g = golden("matris")
    t = f"matris_s{seed}"
    graph = MatRISGraph.from_arrays(g[f"{t}_positions"], g[f"{t}_cell"], g[f"{t}_numbers"], g[f"{t}_edge_index"],
                                    g[f"{t}_edge_image"], g[f"{t}_d2u"], g[f"{t}_u2d"], g[f"{t}_line_graph"],
                                    device=cuda)
    energy, forces, stress = model.energy_forces_stress(graph)
    torch.cuda.synchronize()
    _check(g, seed, energy, forces, stress, e_tol)
    # the energy alone (no backward) is the same number
    assert float(model.energy(graph)[0]) == float(energy[0])


def _builder(g, seed, cuda, **kw):
    from fastmd_b200.graph import FixedCapacityGraphBuilder

    t = f"matris_s{seed}"
    opts = dict(u_capacity=1100, t_capacity=19_000, n_dummy=4)
    opts.update(kw)
    return FixedCapacityGraphBuilder(cell=torch.tensor(g[f"{t}_cell"]), atomic_numbers=torch.tensor(g[f"{t}_numbers"]),
                                     atom_graph_cutoff=6.0, line_graph_cutoff=4.5, candidate_cutoff=8.0, device=cuda,
                                     **opts)


@pytest.mark.parametrize("seed", [0, 1])
def test_matris_on_the_fixed_capacity_graph(cuda, model, seed):
    """This build's fixed-capacity bond graph (sink padding on 4 sink atoms, capacity rows past the real
    ones) gives the result of the reference's legacy graph."""
    g = golden("matris")
    t = f"matris_s{seed}"
    builder = _builder(g, seed, cuda)
    batch, status = builder.build(torch.from_numpy(g[f"{t}_positions"]).to(cuda))
    torch.cuda.synchronize()
    assert int(status.flags.item()) == 0
    assert int(batch.n_edges.item()) == g[f"{t}_edge_index"].shape[0]
    assert int(builder.n_triplets.item()) == g[f"{t}_line_graph"].shape[0]
    energy, forces, stress = model.energy_forces_stress(batch)
    torch.cuda.synchronize()
    assert forces.shape == (135, 3)
    _check(g, seed, energy, forces, stress)


def test_matris_capacity_padding_changes_nothing(cuda, model):
    """More capacity rows (padding edges, bonds and triplets on sink atoms) leave the result bitwise equal."""
    g = golden("matris")
    pos = torch.from_numpy(g["matris_s0_positions"]).to(cuda)
    out = []
    for u_cap, t_cap, n_dummy in ((1100, 19_000, 4), (1400, 24_000, 9)):
        batch, status = _builder(g, 0, cuda, u_capacity=u_cap, t_capacity=t_cap, n_dummy=n_dummy).build(pos)
        out.append(model.energy_forces_stress(batch))
    torch.cuda.synchronize()
    assert float(out[0][0][0]) == pytest.approx(float(out[1][0][0]), rel=1e-12, abs=0)
    assert torch.allclose(out[0][1], out[1][1], rtol=0, atol=1e-9)


T = 500.0


def _md(cuda, seeds=(0,), steps_per_launch=5, skin=2.0):
    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.structures import perovskite
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    systems = [perovskite(seed=s) for s in seeds]
    _, cell, numbers, masses = systems[0]
    momenta = np.concatenate([maxwell_boltzmann_momenta(masses, T, seed=s) for s in seeds])
    return GPUResidentMolecularDynamics(_model(cuda), positions=np.concatenate([s[0] for s in systems]),
                                        momenta=momenta, cell=cell, atomic_numbers=numbers, masses=masses,
                                        temperature_K=T, timestep=0.25 * units.fs, tdamp=25 * units.fs,
                                        replicas=len(seeds), skin=skin, steps_per_launch=steps_per_launch,
                                        device=cuda)


def test_matris_whole_step_trajectory_matches_cpu_oracle(cuda):
    """Config 0's system under MatRIS-10M in whole-step CUDA-graph MD (NVT NHC) against the CPU oracle MD
    (FP64 MatRIS forces, the NHC step in ASE's order) over 10 steps."""
    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.structures import perovskite
    from oracle.md import MatRISOracleMD

    md = _md(cuda)
    steps = 10
    md.run(steps)
    pos, cell, numbers, masses = perovskite(seed=0)
    ref = MatRISOracleMD(seeded_parameters(MATRIS_10M, 0), MATRIS_10M, pos, cell, numbers, masses,
                         maxwell_boltzmann_momenta(masses, T, 0), temperature_K=T, timestep=0.25 * units.fs,
                         tdamp=25 * units.fs)
    for _ in range(steps):
        ref.step()
    q = md.integrator.state.q.cpu().numpy()
    p = md.integrator.state.p.cpu().numpy()
    assert np.abs(q - ref.nhc.q).max() < 1e-6
    assert np.abs(p - ref.nhc.p).max() < 1e-5 * np.abs(ref.nhc.p).max()
    assert abs(float(md.integrator.state.energy[0]) - ref.nhc.E) < 1e-5 * abs(ref.nhc.E)


def test_matris_graph_replay_equals_eager_window(cuda):
    md = _md(cuda)
    integ, runner = md.integrator, md.runner
    snap = integ.snapshot()
    runner._window_body()
    eager = integ.state.flat.clone()
    integ.load_snapshot(snap)
    runner.launch()
    torch.cuda.synchronize()
    assert torch.equal(integ.state.flat, eager)


def test_matris_replica_union_matches_single_systems(cuda):
    """Two replicas as one disjoint union (one graph, per-replica energies) against each run alone."""
    union = _md(cuda, seeds=(0, 1))
    union.run(5)
    n3 = 135 * 3
    for r, seed in enumerate((0, 1)):
        single = _md(cuda, seeds=(seed,))
        single.run(5)
        q_u = union.integrator.state.q.reshape(-1)[r * n3:(r + 1) * n3]
        assert torch.allclose(q_u, single.integrator.state.q.reshape(-1), rtol=0, atol=1e-9)
        assert float(union.integrator.state.energy[r]) == pytest.approx(float(single.integrator.state.energy[0]),
                                                                        rel=1e-9)
