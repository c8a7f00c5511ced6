"""The OpDispatcher mirror (fastmd/engine/dispatch.py:142) on a MatRIS-shaped graph dict: every method
against the oracle of the op it routes to.

Bars: pair maps, gathers and the residual bitwise; segment sums 1e-5 (the oracle sums in float64);
segment attention rtol/atol 2e-6 (exp/log vs NumPy); the identity target CSR bitwise equal to the
permuted CSR of the same (sorted) rows."""
import numpy as np
import pytest
import torch

from oracle import ops as oops
from oracle import pair_aggregate as opa
from oracle import residual_add as ora
from oracle import segment_attention as osa

pytestmark = pytest.mark.gpu


def _graph(n_atoms=57, n_pairs=400, dim=64, seed=0, sorted_target=False):
    rng = np.random.default_rng(seed)
    e = 2 * n_pairs
    d2u = np.repeat(np.arange(n_pairs), 2)[rng.permutation(e)]
    target = rng.integers(0, n_atoms, e)
    if sorted_target:
        target = np.sort(target)
    source = rng.integers(0, n_atoms, e)
    counts = np.bincount(target, minlength=n_atoms)
    graph = {"num_undirected": n_pairs, "num_segment": n_atoms, "_topology_graph_kind": "atom",
             "source_index": torch.from_numpy(source).cuda(), "target_index": torch.from_numpy(target).cuda(),
             "source_bincount": torch.from_numpy(np.bincount(source, minlength=n_atoms)).cuda(),
             "target_bincount": torch.from_numpy(counts).cuda(),
             "_target_segment_attention_counts": torch.from_numpy(counts).cuda()}
    return graph, d2u, source, target, rng


def test_pair_maps_and_residual():
    from fastmd_b200.dispatch import OpDispatcher

    ops = OpDispatcher()
    graph, d2u, _, _, rng = _graph()
    u, dim = graph["num_undirected"], 64
    pair = np.argsort(d2u, kind="stable").reshape(u, 2)
    t_d2u = torch.from_numpy(d2u).cuda()
    data = rng.standard_normal((2 * u, dim)).astype(np.float32)
    x = torch.from_numpy(data).cuda().requires_grad_(True)
    avg = ops.pair_average(x, t_d2u, graph)
    np.testing.assert_array_equal(avg.detach().cpu().numpy(), opa.average(data, pair))
    g = rng.standard_normal((u, dim)).astype(np.float32)
    avg.backward(torch.from_numpy(g).cuda())
    np.testing.assert_array_equal(x.grad.cpu().numpy(), opa.average_bwd(g, pair, 2 * u))
    und = rng.standard_normal((u, dim)).astype(np.float32)
    exp = ops.pair_expand(torch.from_numpy(und).cuda(), t_d2u, graph)
    np.testing.assert_array_equal(exp.cpu().numpy(), opa.expand(und, pair, 2 * u))
    d, r, w = (rng.standard_normal(s).astype(np.float32) for s in ((2 * u, dim), (2 * u, dim), dim))
    res = ops.residual(torch.from_numpy(d).cuda(), torch.from_numpy(r).cuda(), torch.from_numpy(w).cuda())
    np.testing.assert_array_equal(res.cpu().numpy(), ora.forward(d, r, w))


def test_segment_sums():
    from fastmd_b200.dispatch import OpDispatcher

    ops = OpDispatcher()
    graph, _, source, target, rng = _graph(seed=1)
    n, e = graph["num_segment"], len(target)
    value = rng.standard_normal((e, 64)).astype(np.float32)
    weight = rng.standard_normal((e, 64)).astype(np.float32)
    v, w = torch.from_numpy(value).cuda(), torch.from_numpy(weight).cuda()
    for side, seg in (("source", source), ("target", target)):
        got = ops.segment_sum_graph(v, graph[f"{side}_index"], n, graph, side)
        np.testing.assert_allclose(got.cpu().numpy(), oops.segment_sum(value, seg, n), rtol=1e-5, atol=1e-5)
        got = ops.segment_sum_graph(v, graph[f"{side}_index"], n, graph, side, weight=w)
        np.testing.assert_allclose(got.cpu().numpy(), oops.segment_sum(value, seg, n, weight), rtol=1e-5, atol=1e-5)
    assert "_source_segment_sum_csr" in graph and "_target_segment_sum_csr" in graph
    got = ops.segment_sum(v, graph["target_index"], n, weight=w)
    np.testing.assert_allclose(got.cpu().numpy(), oops.segment_sum(value, target, n, weight), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("paired", [True, False])
def test_segment_attention_both_sides(paired):
    from fastmd_b200.dispatch import OpDispatcher

    ops = OpDispatcher(paired_attention=paired)
    graph, _, source, target, rng = _graph(seed=2)
    n, e = graph["num_segment"], len(target)
    la, lb, value = (rng.standard_normal((e, 64)).astype(np.float32) * 3 for _ in range(3))
    v = torch.from_numpy(value).cuda()
    out_s, out_t = ops.segment_attention(torch.from_numpy(la).cuda(), v, graph["source_index"],
                                         torch.from_numpy(lb).cuda(), v, graph["target_index"], n, graph)
    for got, logits, seg in ((out_s, la, source), (out_t, lb, target)):
        perm, off = oops.segment_csr(seg, n)
        ref = osa.forward(logits, value, perm, off)[0]
        np.testing.assert_allclose(got.detach().cpu().numpy(), ref, rtol=2e-6, atol=2e-6)


def test_identity_target_csr_equals_the_permuted_csr():
    from fastmd_b200.dispatch import OpDispatcher

    graph_a, _, _, target, rng = _graph(seed=3, sorted_target=True)
    graph_b = dict(graph_a)
    n, e = graph_a["num_segment"], len(target)
    la, lb, value = (torch.from_numpy(rng.standard_normal((e, 32)).astype(np.float32)).cuda() for _ in range(3))
    ident = OpDispatcher(identity_target_csr={"atom"})
    plain = OpDispatcher()
    a = ident.segment_attention(la, value, graph_a["source_index"], lb, value, graph_a["target_index"], n, graph_a)
    b = plain.segment_attention(la, value, graph_b["source_index"], lb, value, graph_b["target_index"], n, graph_b)
    assert "_target_segment_attention_perm" not in graph_a and "_target_segment_attention_perm" in graph_b
    assert torch.equal(a[1], b[1]) and torch.equal(a[0], b[0])
    sa = ident.segment_sum_graph(value, graph_a["target_index"], n, graph_a, "target")
    sb = plain.segment_sum_graph(value, graph_b["target_index"], n, graph_b, "target")
    assert graph_a["_target_segment_sum_csr"][2] and not graph_b["_target_segment_sum_csr"][2]
    assert torch.equal(sa, sb)


def test_gathers():
    from fastmd_b200.dispatch import OpDispatcher

    ops = OpDispatcher()
    rng = np.random.default_rng(4)
    rows, n = 500, 60
    aligned = rng.standard_normal((rows, 32)).astype(np.float32)
    ga = rng.standard_normal((n, 32)).astype(np.float32)
    gb = rng.standard_normal((n, 16)).astype(np.float32)
    ia, ib, ic = (rng.integers(0, n, rows) for _ in range(3))
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    np.testing.assert_array_equal(ops.gather(t(ga), t(ia)).cpu().numpy(), ga[ia])
    got3 = ops.gather_cat(t(aligned), [t(ga)], [t(ia), t(ib)])
    np.testing.assert_array_equal(got3.cpu().numpy(), oops.aligned_gather_cat3(aligned, ga, ia, ib))
    got4 = ops.gather_cat(t(aligned), [t(ga), t(ga)], [t(ia), t(ib), t(ic)])
    np.testing.assert_array_equal(got4.cpu().numpy(), oops.aligned_gather_cat4(aligned, ga, ia, ga, ib, ic))
    mixed = ops.gather_cat(t(aligned), [t(ga), t(gb)], [t(ia), t(ib), t(ic)])
    ref = oops.gather_cat([(aligned, None), (ga, ia), (gb, ib), (gb, ic)], rows)
    np.testing.assert_array_equal(mixed.cpu().numpy(), ref)
