"""The fixed-capacity MatRIS bond graph (fmd_bond_graph through FixedCapacityGraphBuilder with a line
graph) against the reference builder's own outputs and the oracle.

Bar: bitwise (integer rows, pairs and triplets; the short-edge test is the re-filter's FP32 predicate)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import bond_graph as obg
from oracle import neighbors as onb

pytestmark = pytest.mark.gpu
TAGS = ["perov_sink", "perov_loop", "perov_sink_tover", "perov_loop_eover", "tric_sink"]


def _builder(cell, n_atoms, u_cap, t_cap, sink, n_dummy, cuda, replicas=1):
    from fastmd_b200.graph import FixedCapacityGraphBuilder, PaddingRule

    return FixedCapacityGraphBuilder(
        cell=torch.as_tensor(cell, dtype=torch.float32), atomic_numbers=torch.full((n_atoms,), 14),
        u_capacity=u_cap, t_capacity=t_cap, atom_graph_cutoff=6.0, line_graph_cutoff=4.5, candidate_cutoff=8.0,
        padding=PaddingRule("sink_atoms" if sink else "far_self_loops"), n_dummy=n_dummy, device=cuda,
        replicas=replicas)


def _published(b):
    batch = b.batch
    return dict(center=batch.edge_index[:, 0].cpu().numpy(), neighbor=batch.edge_index[:, 1].cpu().numpy(),
                images=batch.edge_image.cpu().numpy().round().astype(np.int64),
                d2u=batch.directed2undirected.cpu().numpy(), u2d=batch.undirected2directed.cpu().numpy(),
                line_graph=batch.line_graph.cpu().numpy())


@pytest.mark.parametrize("tag", TAGS)
def test_matches_the_reference_builder(cuda, tag):
    from fastmd_b200.graph import fixed_capacity_exceeded

    g = golden("bond_graph")
    N, n_dummy, u_cap, t_cap, total, t_real, sink = (int(v) for v in g[f"bg_{tag}_meta"])
    b = _builder(g[f"bg_{tag}_cell"], N, u_cap, t_cap, bool(sink), n_dummy, cuda)
    if not sink:
        assert tuple(b.pad_image) == tuple(g[f"bg_{tag}_pad_image"])
    _, status = b.build(torch.from_numpy(g[f"bg_{tag}_positions"]).to(cuda))
    got = _published(b)
    for key in ("center", "neighbor", "images", "d2u", "u2d", "line_graph"):
        np.testing.assert_array_equal(got[key], g[f"bg_{tag}_{key}"], err_msg=key)
    overflow, invalid = g[f"bg_{tag}_flags"].tolist()
    assert bool(status.overflow) == bool(overflow) and bool(status.invalid_pairs) == bool(invalid)
    assert int(status.edge_count.item()) == total and int(status.triplet_count.item()) == t_real
    assert bool(fixed_capacity_exceeded(status, b)) == bool(overflow)
    if overflow:  # grown capacities fit
        grown = b.resized(u_cap + 64, t_real + 256)
        _, st = grown.build(torch.from_numpy(g[f"bg_{tag}_positions"]).to(cuda))
        assert not bool(st.overflow) and not bool(fixed_capacity_exceeded(st, grown))


def _union_oracle(pos, cell, replicas, u_cap, t_cap, n_dummy):
    """The oracle bond graph of a union of ``replicas`` copies (edges of each copy, atom ids offset)."""
    n = pos.shape[0] // replicas
    parts = []
    for r in range(replicas):
        p = pos[r * n:(r + 1) * n]
        wrapped, _, _ = onb.wrap(p, cell, inv_cell=onb.inverse_cell(cell))
        c, nb, im, _, short = onb.refilter(wrapped, cell, *onb.candidates(wrapped, cell, 8.0), 6.0, line_cutoff=4.5)
        parts.append((c + r * n, nb + r * n, im, short))
    c, nb, im, short = (np.concatenate(x) for x in zip(*parts))
    return obg.build(c, nb, im, short, c.size, n_real=pos.shape[0], u_capacity=u_cap, t_capacity=t_cap, sink=True,
                     n_dummy=n_dummy)


def test_replica_union_equals_the_oracle(cuda):
    from fastmd_b200.structures import perovskite

    R = 6
    pos = np.concatenate([perovskite(seed=s)[0] for s in range(R)]).astype(np.float32)
    cell = perovskite(seed=0)[1]
    b = _builder(cell, pos.shape[0] // R, 1060 * R, 19_000 * R, True, 64, cuda, replicas=R)
    _, status = b.build(torch.from_numpy(pos).to(cuda))
    ref = _union_oracle(pos, cell, R, 1060 * R, 19_000 * R, 64)
    assert not bool(status.overflow) and not ref["overflow"]
    got = _published(b)
    for key in ("center", "neighbor", "images", "d2u", "u2d", "line_graph"):
        np.testing.assert_array_equal(got[key], ref[key], err_msg=key)
    assert int(status.triplet_count.item()) == ref["n_triplets"]


def test_capture_replay_equals_eager_builds(cuda):
    """The build is capture-safe: a CUDA graph of it, replayed on moved positions, publishes exactly what an
    eager build of the same positions does (candidates reused, no host read)."""
    from fastmd_b200.structures import perovskite

    pos, cell, _, _ = perovskite(seed=0)
    n = pos.shape[0]
    eager = _builder(cell, n, 1100, 19_000, True, 64, cuda)
    graphed = _builder(cell, n, 1100, 19_000, True, 64, cuda)
    start = torch.from_numpy(pos.astype(np.float32)).to(cuda)
    eager.refresh_candidates(start)
    graphed.refresh_candidates(start)
    buf = start.clone()
    graphed.build(buf, rebuild_candidates=False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        graphed.build(buf, rebuild_candidates=False)
    rng = np.random.default_rng(3)
    for _ in range(3):
        moved = start + torch.from_numpy(rng.normal(0, 0.05, pos.shape).astype(np.float32)).to(cuda)
        buf.copy_(moved)
        graph.replay()
        eager.build(moved, rebuild_candidates=False)
        a, b = _published(graphed), _published(eager)
        for key in a:
            np.testing.assert_array_equal(a[key], b[key], err_msg=key)
        assert int(graphed.flags.item()) == int(eager.flags.item())
    graph.reset()


def test_bond_graph_invariants_at_a_large_union(cuda):
    """64 replicas (8,640 atoms, ~131k edges, ~1.1M triplets): every real pair maps back, every triplet's
    two edges leave its atom and are short, the padded rows are sinks."""
    from fastmd_b200.structures import perovskite

    R = 64
    pos = np.concatenate([perovskite(seed=s)[0] for s in range(R)]).astype(np.float32)
    cell = perovskite(seed=0)[1]
    n_real = pos.shape[0]
    b = _builder(cell, n_real // R, 1060 * R, 19_000 * R, True, 64, cuda, replicas=R)
    _, status = b.build(torch.from_numpy(pos).to(cuda))
    assert int(status.flags.item()) == 0
    E, T = int(status.edge_count.item()), int(status.triplet_count.item())
    batch = b.batch
    ei, d2u, u2d = batch.edge_index.long(), batch.directed2undirected.long(), batch.undirected2directed.long()
    U = E // 2
    assert torch.equal(d2u[u2d[:U]], torch.arange(U, device=cuda))
    img = batch.edge_image
    partner = torch.full((U, 2), -1, dtype=torch.long, device=cuda)
    rows = torch.arange(E, device=cuda)
    first = u2d[d2u[:E]] == rows
    partner[d2u[:E][first], 0] = rows[first]
    partner[d2u[:E][~first], 1] = rows[~first]
    a, c = partner[:, 0], partner[:, 1]
    assert torch.all(c >= 0) and torch.equal(ei[a, 0], ei[c, 1]) and torch.equal(ei[a, 1], ei[c, 0])
    assert torch.equal(img[a], -img[c])
    lg = batch.line_graph[:T].long()
    assert torch.equal(ei[lg[:, 2], 0], lg[:, 0]) and torch.equal(ei[lg[:, 4], 0], lg[:, 0])
    assert torch.equal(d2u[lg[:, 2]], lg[:, 1]) and torch.equal(d2u[lg[:, 4]], lg[:, 3])
    assert torch.all(lg[:, 2] != lg[:, 4])
    wrapped = batch.positions[:n_real]
    for col in (2, 4):
        e = lg[:, col]
        vec = wrapped[ei[e, 1]] - wrapped[ei[e, 0]] + img[e] @ b.cell
        assert float(vec.norm(dim=1).max()) < 4.5 + 1e-4
    assert torch.all(ei[E:] >= n_real)
