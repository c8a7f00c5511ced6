"""Long-run NVT statistics of config 1 (the 135-atom perovskite, MACE-architecture potential, NHC at 500 K,
dt 0.25 fs, tdamp 25 fs) in whole-step CUDA-graph MD.

* 10,000 GPU steps (2.5 ps): the drift of the NHC conserved energy (the fitted slope, gpu_nhc.py:1231
  ``conserved_energy``) stays below 1e-4 eV/ps per atom (measured on a B200: 1.1e-5) and its spread below
  2e-4 eV per atom (measured 2.2e-5); over the last 80 % of the run the mean temperature is within 25 K of
  500 K and its standard deviation within 0.6-1.4 of the canonical sqrt(2 / 3N) T = 35.1 K (measured
  503 K and 29.9 K).
* the first 1,000 steps against the CPU oracle MD (FP64 forces, the NHC in ASE's operation order) over the
  same 1,000 steps: the GPU drift is no worse than twice the oracle's (+1e-5 eV/ps; measured -3.8e-5 vs
  -3.1e-5 eV/ps), the conserved energies agree within 1e-4 eV (measured 1.0e-5) and the mean temperatures
  within 0.01 K.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

T, N, DT_PS = 500.0, 135, 0.25e-3


def _slope(t, y):
    return float(np.polyfit(t, y, 1)[0])


def test_config1_long_nvt_statistics(cuda):
    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.mace import MACEConfig, MACEModel, init_weights
    from fastmd_b200.structures import perovskite
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics
    from oracle.md import OracleMD

    pos, cell, numbers, masses = perovskite(seed=0)
    momenta = maxwell_boltzmann_momenta(masses, T, 0)
    md = GPUResidentMolecularDynamics(MACEModel(device=cuda, seed=1), positions=pos, momenta=momenta, cell=cell,
                                      atomic_numbers=numbers, masses=masses, temperature_K=T,
                                      timestep=0.25 * units.fs, tdamp=25 * units.fs, steps_per_launch=10,
                                      device=cuda)
    conserved, temps = [], []
    for _ in range(1000):
        md.run(10)
        th = md.thermodynamics()
        conserved.append(float(th["conserved_energy"][0]))
        temps.append(float(th["temperature"][0]))
    conserved, temps = np.array(conserved), np.array(temps)
    t_ps = np.arange(1, 1001) * 10 * DT_PS
    assert abs(_slope(t_ps, conserved)) / N < 1e-4
    assert (conserved.max() - conserved.min()) / N < 2e-4
    tail = temps[200:]
    canonical = T * np.sqrt(2.0 / (3 * N))
    assert abs(tail.mean() - T) < 25.0
    assert 0.6 * canonical < tail.std() < 1.4 * canonical

    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = OracleMD(init_weights(MACEConfig(), 1), MACEConfig(), pos, cell, numbers, masses, momenta,
                   temperature_K=T, timestep=0.25 * units.fs, tdamp=25 * units.fs)
    oc, ot = [], []
    for step in range(1000):
        ref.step()
        if (step + 1) % 10 == 0:
            oc.append(ref.nhc.conserved_energy())
            ot.append(ref.nhc.temperature())
    oc = np.array(oc)
    gpu_drift, ref_drift = _slope(t_ps[:100], conserved[:100]), _slope(t_ps[:100], oc)
    assert abs(gpu_drift) <= 2.0 * abs(ref_drift) + 1e-5
    assert np.abs(conserved[:100] - oc).max() < 1e-4
    assert abs(temps[:100].mean() - np.mean(ot)) < 0.01
