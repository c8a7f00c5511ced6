"""The float64 edges-only build (positions_dtype=torch.float64, fixed_capacity_builder.py:2315) against the
reference prologue's golden outputs: float64 model positions, float32 wrap, wrap delta and skin test bitwise;
the edges are those of the float32 build of the rounded coordinates."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _builder(cell64, n, cuda, dtype=torch.float64, u_capacity=8192):
    from fastmd_b200.graph import FixedCapacityGraphBuilder

    return FixedCapacityGraphBuilder(cell=torch.from_numpy(np.asarray(cell64, np.float64)),
                                     atomic_numbers=torch.full((n,), 14), u_capacity=u_capacity, atom_graph_cutoff=6.0,
                                     candidate_cutoff=8.0, device=cuda, positions_dtype=dtype)


@pytest.mark.parametrize("tag", ["tric", "cubic"])
def test_float64_prologue_matches_the_reference(cuda, tag):
    g = golden("float64")
    cell64, pos64, ref64 = g[f"f64_{tag}_cell"], g[f"f64_{tag}_positions"], g[f"f64_{tag}_reference"]
    n = pos64.shape[0]
    b = _builder(cell64, n, cuda)
    b.refresh_candidates(torch.from_numpy(ref64).to(cuda))
    np.testing.assert_array_equal(b.reference_wraps.cpu().numpy(), g[f"f64_{tag}_ref_wraps"])
    batch, status = b.build(torch.from_numpy(pos64).to(cuda), rebuild_candidates=False)
    assert batch.positions.dtype == torch.float64 and batch.cell.dtype == torch.float64
    np.testing.assert_array_equal(batch.positions.cpu().numpy(), g[f"f64_{tag}_model_positions"])
    np.testing.assert_array_equal(b.wrapped32.cpu().numpy(), g[f"f64_{tag}_wrapped"])
    np.testing.assert_array_equal(b.wrap_delta.cpu().numpy(), g[f"f64_{tag}_wrap_delta"])
    assert float(b.max_displacement[0]) == float(g[f"f64_{tag}_max_displacement"][0])
    assert bool(status.candidate_valid) == bool(g[f"f64_{tag}_candidate_valid"][0])
    # the edges: those of the float32 build of the rounded coordinates, bitwise
    b32 = _builder(cell64, n, cuda, dtype=torch.float32)
    b32.refresh_candidates(torch.from_numpy(ref64.astype(np.float32)).to(cuda))
    batch32, _ = b32.build(torch.from_numpy(pos64.astype(np.float32)).to(cuda), rebuild_candidates=False)
    assert torch.equal(batch.n_edges, batch32.n_edges)
    assert torch.equal(batch.edge_index, batch32.edge_index) and torch.equal(batch.edge_image, batch32.edge_image)
    np.testing.assert_array_equal(b.wrapped32.cpu().numpy(), batch32.positions.cpu().numpy())
    if bool(status.candidate_valid):
        # every real edge is within the cutoff in float64 too (the images agree with the float64 positions)
        E = int(batch.n_edges.item())
        ei = batch.edge_index[:E].long()
        vec = batch.positions[ei[:, 1]] - batch.positions[ei[:, 0]] + batch.edge_image[:E].double() @ batch.cell
        assert float(vec.norm(dim=1).max()) < 6.0 + 1e-5
