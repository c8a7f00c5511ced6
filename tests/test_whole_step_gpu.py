"""Whole-step CUDA-graph MD: the captured window against eager steps and the CPU oracle MD."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

T = 500.0


def _md(cuda, *, seeds=(0,), skin=2.0, steps_per_launch=5, channels=128, execution="whole_step"):
    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.mace import MACEConfig, MACEModel
    from fastmd_b200.structures import perovskite
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    systems = [perovskite(seed=s) for s in seeds]
    _, cell, numbers, masses = systems[0]
    momenta = np.concatenate([maxwell_boltzmann_momenta(masses, T, seed=s) for s in seeds])
    model = MACEModel(MACEConfig(channels=channels), device=cuda, seed=1)
    return GPUResidentMolecularDynamics(model, positions=np.concatenate([s[0] for s in systems]), momenta=momenta,
                                        cell=cell,
                                        atomic_numbers=numbers, masses=masses, temperature_K=T,
                                        timestep=0.25 * units.fs, tdamp=25 * units.fs, replicas=len(seeds),
                                        skin=skin, steps_per_launch=steps_per_launch, execution=execution,
                                        device=cuda)


def test_trajectory_matches_cpu_oracle(cuda):
    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.structures import perovskite
    from oracle.md import OracleMD

    md = _md(cuda)
    steps = 20
    md.run(steps)
    pos, cell, numbers, masses = perovskite(seed=0)
    ref = OracleMD(md.model.weights_host, md.model.config, pos, cell, numbers, masses,
                   maxwell_boltzmann_momenta(masses, T, 0), temperature_K=T, timestep=0.25 * units.fs,
                   tdamp=25 * units.fs)
    for _ in range(steps):
        ref.step()
    q = md.integrator.state.q.cpu().numpy()
    p = md.integrator.state.p.cpu().numpy()
    assert np.abs(q - ref.nhc.q).max() < 1e-6
    assert np.abs(p - ref.nhc.p).max() < 1e-5 * np.abs(ref.nhc.p).max()
    e = float(md.integrator.state.energy[0])
    assert abs(e - ref.nhc.E) < 1e-7 * abs(ref.nhc.E)
    assert abs(float(md.integrator.temperature()) - ref.nhc.temperature()) < 1e-6 * ref.nhc.temperature()


def test_graph_replay_bitwise_equals_eager_window(cuda):
    md = _md(cuda)
    integ, runner = md.integrator, md.runner
    snap = integ.snapshot()
    runner._window_body()
    eager = integ.state.flat.clone()
    integ.load_snapshot(snap)
    runner.launch()
    torch.cuda.synchronize()
    assert torch.equal(integ.state.flat, eager)


def test_skin_fallbacks_keep_the_exact_trajectory(cuda):
    """A skin too small for the window forces rollbacks and candidate refreshes; the edges are exact
    either way, so the trajectory equals the large-skin one bit for bit."""
    small = _md(cuda, skin=0.004)
    large = _md(cuda, skin=2.0)
    small.run(20)
    large.run(20)
    assert small.runner.fallbacks > 0
    assert torch.equal(small.integrator.state.flat, large.integrator.state.flat)


def test_replica_md_equals_single_runs(cuda):
    union = _md(cuda, seeds=(0, 1))
    union.run(10)
    n3 = 135 * 3
    for r in (0, 1):
        single = _md(cuda, seeds=(r,))
        single.run(10)
        st = single.integrator.state
        assert torch.equal(union.integrator.state.q.reshape(-1)[r * n3:(r + 1) * n3], st.q.reshape(-1))
        assert torch.equal(union.integrator.state.p.reshape(-1)[r * n3:(r + 1) * n3], st.p.reshape(-1))
        assert torch.equal(union.integrator.state.energy[r], st.energy[0])


def test_execution_modes_give_one_trajectory(cuda):
    """model_graph (bucket replays of ragged builds) and eager give the same trajectory bit for bit, and
    the whole-step windows (fixed-capacity builds) the same one to rounding of the edge order."""
    steps = 10
    runs = {}
    for execution in ("model_graph", "eager", "whole_step"):
        md = _md(cuda, execution=execution)
        md.run(steps)
        runs[execution] = md
    mg, eg, ws = (runs[k].integrator.state for k in ("model_graph", "eager", "whole_step"))
    assert torch.equal(mg.flat, eg.flat)
    assert (mg.q - ws.q).abs().max().item() < 1e-9
    assert runs["model_graph"].runner.stats()["captures"] >= 1
    with pytest.raises(RuntimeError):
        runs["eager"].step_host(None, None, {})


@pytest.mark.parametrize("execution", ["whole_step", "model_graph"])
def test_restart_continues_the_trajectory_bitwise(cuda, tmp_path, execution):
    """10 steps, a restart file, 10 more steps; a fresh driver loaded from the file runs the same 10 steps
    to the same state bit for bit (the cached forces are not re-evaluated); frames read back."""
    from fastmd_b200.md_protocol import ExtxyzTrajectory, read_extxyz, read_restart, write_restart

    a = _md(cuda, execution=execution)
    a.run(10)
    write_restart(tmp_path / "r.npz", a.restart_data(parameters={"note": "test"}))
    traj = ExtxyzTrajectory(tmp_path / "t.extxyz")
    a.write_frame(traj)
    a.run(10)
    a.write_frame(traj)
    traj.close()
    data = read_restart(tmp_path / "r.npz")
    assert data.step == 10 and data.engine == "native" and data.parameters["note"] == "test"
    b = _md(cuda, execution=execution, seeds=(5,))  # another start, overwritten by the file
    b.load_restart(data)
    b.run(10)
    assert b.steps_done == 20
    assert torch.equal(a.integrator.state.flat, b.integrator.state.flat)
    frames = read_extxyz(tmp_path / "t.extxyz")
    assert [f["step"] for f in frames] == [10, 20]
    q = a.integrator.state.q.cpu().numpy()
    assert np.abs(frames[1]["positions"] - q).max() < 1e-7
