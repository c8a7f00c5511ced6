"""Edge cases of the step path on the GPU: builds without a single pair (a sparse box, one atom), the
fused model on them (energies are the element references plus the readout of the embedding alone,
forces exactly zero), their model_graph replay, and empty segment sums."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _sparse(cuda, n=4, box=40.0):
    """n atoms on a diagonal, 10 A apart in a 40 A box: no pair within 6 A."""
    pos = np.array([[10.0 * i, 10.0 * i, 10.0 * i] for i in range(n)], np.float32) % box
    cell = np.eye(3, dtype=np.float32) * box
    numbers = np.array([55, 50, 53, 53][:n])
    return pos, cell, numbers


def test_ragged_list_without_pairs(cuda):
    from fastmd_b200.graph import TensorGraphBuilder, neighbor_list

    pos, cell, numbers = _sparse(cuda)
    center, neighbor, images, dist = neighbor_list(torch.from_numpy(pos).to(cuda), torch.from_numpy(cell), 6.0)
    assert center.shape[0] == 0 and neighbor.shape[0] == 0 and images.shape == (0, 3) and dist.shape[0] == 0
    b = TensorGraphBuilder(cell=torch.from_numpy(cell), atomic_numbers=torch.from_numpy(numbers), device=cuda)
    batch = b.build(torch.from_numpy(pos).to(cuda))
    assert batch.edge_index.shape == (0, 2) and int(batch.n_edges.item()) == 0
    assert torch.equal(batch.recv_off.cpu(), torch.zeros(len(numbers) + 1, dtype=torch.int64))


@pytest.mark.parametrize("n", [1, 4])
def test_fused_model_on_a_graph_without_edges(cuda, n):
    from oracle import mace as omace

    from fastmd_b200.graph import TensorGraphBuilder
    from fastmd_b200.mace import MACEModel
    from fastmd_b200.model_graph import BucketedGraphRunner

    pos, cell, numbers = _sparse(cuda, n)
    b = TensorGraphBuilder(cell=torch.from_numpy(cell), atomic_numbers=torch.from_numpy(numbers), device=cuda)
    batch = b.build(torch.from_numpy(pos).to(cuda))
    model = MACEModel(device=cuda)
    energy, forces = (x.clone() for x in model.energy_forces_fused(model.prepare(batch)))
    assert torch.equal(forces, torch.zeros_like(forces))
    E, F, _ = omace.energy_forces(model.weights_host, model.config, pos.astype(np.float64), cell, numbers,
                                  np.zeros((0, 2), np.int64), np.zeros((0, 3)), n_systems=1)
    assert abs(float(energy[0]) - float(np.asarray(E).reshape(-1)[0])) < 1e-7 * max(1.0, abs(float(energy[0])))
    assert np.abs(F).max() == 0.0
    e2, f2 = BucketedGraphRunner(model, u_step=16, min_pad_u=0).run(batch)
    assert torch.equal(e2, energy) and torch.equal(f2, forces)


def test_segment_sum_with_no_rows_and_empty_segments(cuda):
    from fastmd_b200.ops import csr_segment_sum

    v = torch.zeros(0, 8, device=cuda)
    seg = torch.zeros(0, dtype=torch.int64, device=cuda)
    out = csr_segment_sum(v, seg, 5)
    assert out.shape == (5, 8) and torch.count_nonzero(out) == 0
    v = torch.randn(6, 8, device=cuda)
    seg = torch.tensor([0, 0, 3, 3, 3, 4], device=cuda)
    out = csr_segment_sum(v, seg, 6)
    assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[2]) == 0 and torch.count_nonzero(out[5]) == 0
    torch.testing.assert_close(out[3], v[2:5].sum(0), rtol=1e-6, atol=1e-6)


def test_zero_row_inputs_of_the_op_surface(cuda):
    """Every op of the surface takes inputs without rows (an empty graph's edges, a system without bonds)
    and returns the reference's empty results: zeros / -inf lse for the segments, empty rows elsewhere."""
    from fastmd_b200 import gated_ln, line_graph, segment_attention, wide_gemm
    from fastmd_b200.decomposed_indexed_cat_silu_linear import decomposed_indexed_cat3_silu_linear

    D = 16
    z = torch.zeros(0, D, device=cuda)
    seg = torch.zeros(0, dtype=torch.int64, device=cuda)
    out, lse = segment_attention.segment_attention(z, z, seg, 4, return_lse=True)
    assert out.shape == (4, D) and torch.count_nonzero(out) == 0 and torch.isneginf(lse).all()
    pa = segment_attention.paired_segment_attention(z, z, z, seg, seg, 3)
    assert all(t.shape == (3, D) and torch.count_nonzero(t) == 0 for t in pa[:2])
    w = torch.ones(D, device=cuda)
    assert gated_ln.fused_gated_ln(z, z, w, w * 0, w, w * 0).shape == (0, D)
    W = torch.randn(32, D, device=cuda)
    assert wide_gemm.linear(z, W).shape == (0, 32)
    gathered = torch.randn(5, D, device=cuda)
    ws = tuple(torch.randn(8, D, device=cuda) for _ in range(3))
    core, gate = decomposed_indexed_cat3_silu_linear(z, gathered, seg, seg, ws)
    assert core.shape == (0, 4) and gate.shape == (0, 4)
    d2u, u2d = line_graph.build_d2u(seg, seg, torch.zeros(0, 3, dtype=torch.int32, device=cuda), 5)
    assert d2u.shape == (0,) and u2d.shape == (0,)
    trip = line_graph.build_line_graph(seg, d2u, torch.zeros(0, device=cuda), 5, 4.5)
    assert trip.shape == (0, 5)
