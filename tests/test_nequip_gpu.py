"""The NequIP-architecture (SevenNet-0-style, config 3) model on the GPU against the FP64 oracle
(energies unpinned to sevenn, which is absent; the coupling constants are pinned to Racah's formula in
tests/test_nequip_oracle.py). Bars: config 3 itself (5 layers, 5,000 atoms) energy 1e-6 relative and
forces 1e-5 of the largest force; a 3-layer model on the 135-atom cell at the FP32 bar of 1e-5 relative
for both (IEEE and 3xTF32 linears; measured on a B200: energy 2.7e-6 / 3.0e-6, the two paths within
2e-7 of each other, so the gap is the FP32 geometry and radial basis they share, not the linears;
forces 3.7e-6 of the largest); a padded exact-rc build gives the ragged
build's energy and forces bit for bit (the padded rows are at the cutoff, where every radial weight
vanishes, and no CSR visits them)."""
import numpy as np
import pytest
import torch

from oracle import nequip as onq

pytestmark = pytest.mark.gpu


def _ragged(pos, cell, numbers, cuda):
    from fastmd_b200.graph import TensorGraphBuilder

    b = TensorGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32), atomic_numbers=torch.tensor(numbers),
                           atom_graph_cutoff=5.0, device=cuda)
    return b.build(torch.from_numpy(pos.astype(np.float32)).to(cuda))


@pytest.mark.parametrize("precision", ["ieee", "tf32x3"])
def test_matches_the_oracle(cuda, precision):
    from fastmd_b200.nequip import NequIPConfig, NequIPModel
    from fastmd_b200.structures import perovskite

    pos, cell, numbers, _ = perovskite(seed=0)
    config = NequIPConfig(num_layers=3)
    model = NequIPModel(config, device=cuda, precision=precision)
    batch = _ragged(pos, cell, numbers, cuda)
    e, f = model.energy_forces(batch)
    ei = batch.edge_index.cpu().numpy()
    ref_e, ref_f = onq.energy_forces(model.host_weights, config, batch.positions.cpu().numpy().astype(np.float64),
                                     cell, numbers, ei[:, 0], ei[:, 1], batch.edge_image.cpu().numpy())
    assert abs(float(e[0]) - ref_e) <= 1e-5 * abs(ref_e), (float(e[0]), ref_e)
    err = np.abs(f.cpu().numpy() - ref_f).max() / np.abs(ref_f).max()
    assert err < 1e-5, err


@pytest.mark.parametrize("precision", ["ieee", "tf32x3"])
def test_config3_model_matches_the_oracle_at_1e5(cuda, precision):
    """Config 3 itself: the 5-layer 128x0e + 64x1e + 32x2e model (rc 5 A) on the 10 x 10 x 10 ABX3
    supercell (5,000 atoms, 60,000 edges, seed 3) against the FP64 oracle: energy within 1e-6 relative,
    forces within 1e-5 of the largest force (measured on a B200: 6.8e-8 / 6.8e-6 with IEEE linears,
    3.3e-7 / 6.7e-6 with 3xTF32)."""
    from fastmd_b200.nequip import NequIPConfig, NequIPModel
    from fastmd_b200.structures import perovskite

    pos, cell, numbers, _ = perovskite(reps=10, seed=3)
    config = NequIPConfig()
    assert config.num_layers == 5 and config.r_max == 5.0
    model = NequIPModel(config, device=cuda, precision=precision)
    batch = _ragged(pos, cell, numbers, cuda)
    e, f = model.energy_forces(batch)
    ei = batch.edge_index.cpu().numpy()
    ref_e, ref_f = onq.energy_forces(model.host_weights, config, batch.positions.cpu().numpy().astype(np.float64),
                                     cell, numbers, ei[:, 0], ei[:, 1], batch.edge_image.cpu().numpy())
    assert len(numbers) == 5000 and ei.shape[0] > 50_000
    assert abs(float(e[0]) - ref_e) <= 1e-6 * abs(ref_e), (float(e[0]), ref_e)
    assert np.abs(f.cpu().numpy() - ref_f).max() <= 1e-5 * np.abs(ref_f).max()


def test_padded_exact_rc_build_equals_the_ragged_build(cuda):
    from fastmd_b200.graph import FixedCapacityGraphBuilder, PaddingRule
    from fastmd_b200.nequip import NequIPConfig, NequIPModel
    from fastmd_b200.structures import perovskite

    pos, cell, numbers, _ = perovskite(seed=1)
    model = NequIPModel(NequIPConfig(num_layers=2), device=cuda)
    e1, f1 = model.energy_forces(_ragged(pos, cell, numbers, cuda))
    fixed = FixedCapacityGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32),
                                      atomic_numbers=torch.tensor(numbers), u_capacity=1200, atom_graph_cutoff=5.0,
                                      padding=PaddingRule("exact_rc_loops"), device=cuda)
    batch, status = fixed.build(torch.from_numpy(pos.astype(np.float32)).to(cuda))
    assert int(status.flags.item()) == 0 and int(batch.n_edges.item()) < 2400
    e2, f2 = model.energy_forces(batch)
    assert torch.equal(e1, e2) and torch.equal(f1, f2)


def test_md_whole_step_equals_eager(cuda):
    """NVT MD under the NequIP potential: the whole_step mode (windows captured as CUDA graphs, the
    autograd force evaluation inside) gives the eager mode's trajectory bit for bit."""
    from fastmd_b200 import units
    from fastmd_b200.nequip import NequIPConfig, NequIPModel
    from fastmd_b200.structures import perovskite
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    pos, cell, numbers, masses = perovskite(seed=2)
    model = NequIPModel(NequIPConfig(num_layers=2), device=cuda)
    runs = {}
    for execution in ("whole_step", "eager"):
        md = GPUResidentMolecularDynamics(model, positions=pos, cell=cell, atomic_numbers=numbers, masses=masses,
                                          temperature_K=500.0, timestep=0.25 * units.fs, tdamp=25 * units.fs,
                                          steps_per_launch=5, execution=execution, device=cuda)
        md.run(20)
        runs[execution] = md.integrator.state.flat.clone()
    assert torch.equal(runs["whole_step"], runs["eager"])


def test_gate_matches_torch_fp32(cuda):
    """fmd_nequip_gate and its backward against the same expressions in torch FP32 (silu, sigmoid,
    products and sums): values and gradients within 2e-6 relative."""
    from fastmd_b200.nequip import gate

    g = torch.Generator(device="cpu").manual_seed(5)
    n = 1037
    shapes = [(n, 224), (3 * n, 64), (5 * n, 32), (n, 128), (3 * n, 64), (5 * n, 32)]
    ins = [(torch.randn(s, generator=g) * 3).to(cuda).requires_grad_(True) for s in shapes]
    out = gate(*ins)
    ref_in = [t.detach().clone().requires_grad_(True) for t in ins]
    o0, o1, o2, s0, s1, s2 = ref_in
    gates = torch.sigmoid(o0[:, 128:])
    ref = [torch.nn.functional.silu(o0[:, :128]) + s0,
           (o1.view(n, 3, 64) * gates[:, None, :64]).view(3 * n, 64) + s1,
           (o2.view(n, 5, 32) * gates[:, None, 64:]).view(5 * n, 32) + s2]
    for a, b in zip(out, ref):
        assert a.shape == b.shape
        assert torch.allclose(a, b, rtol=2e-6, atol=2e-6)
    up = [torch.randn(t.shape, generator=g).to(cuda) for t in ref]
    grads = torch.autograd.grad(out, ins, up)
    ref_grads = torch.autograd.grad(ref, ref_in, up)
    for a, b in zip(grads, ref_grads):
        assert torch.allclose(a, b, rtol=2e-6, atol=2e-6 * float(b.abs().max())), float((a - b).abs().max())


def test_gate_of_no_atoms_is_a_no_op(cuda):
    from fastmd_b200.nequip import gate

    ins = [torch.zeros(0, w, device=cuda) for w in (224, 64, 32, 128, 64, 32)]
    assert [tuple(t.shape) for t in gate(*ins)] == [(0, 128), (0, 64), (0, 32)]


def test_self_connection_matches_torch_fp32(cuda):
    """fmd_nequip_self_connection (out[n, m] = x[n, m] @ w[elem[n]]) and its input gradient (the same
    kernel on the transposed weights) against torch FP32 einsums: within 1e-5 relative of the largest
    value."""
    from fastmd_b200._lib import call, ptr

    g = torch.Generator(device="cpu").manual_seed(9)
    n, n_elem = 777, 89
    elem = torch.randint(0, n_elem, (n,), generator=g).to(cuda)
    w = [torch.randn(n_elem, u, u, generator=g).to(cuda) / u ** 0.5 for u in (128, 64, 32)]
    wt = [wl.transpose(1, 2).contiguous() for wl in w]
    xs = [torch.randn(n * d, u, generator=g).to(cuda) for d, u in ((1, 128), (3, 64), (5, 32))]

    def self_connection(planes, weights):
        out = [torch.empty_like(t) for t in planes]
        call("fmd_nequip_self_connection", *[ptr(t) for t in planes], ptr(elem), *[ptr(t) for t in weights], n, 0,
             *[ptr(t) for t in out], None)
        return out

    out = self_connection(xs, w)
    ref_x = [t.clone().requires_grad_(True) for t in xs]
    ref = [torch.einsum("nmu,nuv->nmv", t.view(n, d, -1), wl[elem]).reshape(n * d, -1)
           for t, d, wl in zip(ref_x, (1, 3, 5), w)]
    for a, b in zip(out, ref):
        assert (a - b).abs().max() <= 1e-5 * b.abs().max()
    up = [torch.randn(t.shape, generator=g).to(cuda) for t in ref]
    for a, b in zip(self_connection(up, wt), torch.autograd.grad(ref, ref_x, up)):
        assert (a - b).abs().max() <= 1e-5 * b.abs().max()
