"""Gather-cat and CSR segment sums on the GPU against the reference's kernels (golden) and the oracle."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import ops as oops

pytestmark = pytest.mark.gpu


def _t(x, device):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device)


@pytest.mark.parametrize("tag", ["small", "wide", "odd"])
def test_gather_cat3_forward_bitwise_backward_deterministic(cuda, tag):
    from fastmd_b200 import ops

    g = golden("gather_cat")
    A, X, ia, ib, G = (_t(g[f"cat3_{tag}_{k}"], cuda) for k in ("A", "X", "ia", "ib", "G"))
    A.requires_grad_(True)
    X.requires_grad_(True)
    out = ops.aligned_gather_cat3(A, X, ia, ib)
    assert torch.equal(out.detach().cpu(), torch.from_numpy(g[f"cat3_{tag}_out"]))
    ga, gx = torch.autograd.grad(out, (A, X), G)
    assert torch.equal(ga.cpu(), torch.from_numpy(g[f"cat3_{tag}_grad_aligned"]))
    np.testing.assert_allclose(gx.cpu().numpy(), g[f"cat3_{tag}_grad_gathered"], rtol=1e-5, atol=1e-5)
    _, ox = oops.aligned_gather_cat3_bwd(g[f"cat3_{tag}_G"], X.shape[0], g[f"cat3_{tag}_ia"], g[f"cat3_{tag}_ib"])
    np.testing.assert_allclose(gx.cpu().numpy(), ox, rtol=1e-5, atol=1e-5)
    # no atomics: a second backward gives the same bits
    ga2, gx2 = torch.autograd.grad(ops.aligned_gather_cat3(A, X, ia, ib), (A, X), G)
    assert torch.equal(gx, gx2) and torch.equal(ga, ga2)


def test_gather_cat4_matches_reference(cuda):
    from fastmd_b200 import ops

    g = golden("gather_cat")
    A, Xa, Xb, ia, ib, ic, G = (_t(g[f"cat4_{k}"], cuda) for k in ("A", "Xa", "Xb", "ia", "ib", "ic", "G"))
    for t in (A, Xa, Xb):
        t.requires_grad_(True)
    out = ops.aligned_gather_cat4(A, Xa, ia, Xb, ib, ic)
    assert torch.equal(out.detach().cpu(), torch.from_numpy(g["cat4_out"]))
    g0, g1, g2 = torch.autograd.grad(out, (A, Xa, Xb), G)
    assert torch.equal(g0.cpu(), torch.from_numpy(g["cat4_grad_aligned"]))
    np.testing.assert_allclose(g1.cpu().numpy(), g["cat4_grad_a"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(g2.cpu().numpy(), g["cat4_grad_b"], rtol=1e-5, atol=1e-5)


def test_mixed_width_gather_cat_c2_layout(cuda):
    """[X[sender] 128 | X[receiver] 128 | basis 8]: the op-microbenchmark edge row (one kernel)."""
    from fastmd_b200 import ops

    rng = np.random.default_rng(3)
    N, E = 300, 4000
    X = rng.standard_normal((N, 128)).astype(np.float32)
    B = rng.standard_normal((E, 8)).astype(np.float32)
    snd = rng.integers(0, N, E)
    rcv = np.sort(rng.integers(0, N, E))
    Xt, Bt = _t(X, cuda).requires_grad_(True), _t(B, cuda).requires_grad_(True)
    out = ops.gather_cat([(Xt, _t(snd, cuda)), (Xt, _t(rcv, cuda)), (Bt, None)])
    ref = oops.gather_cat([(X, snd), (X, rcv), (B, None)], E)
    assert torch.equal(out.detach().cpu(), torch.from_numpy(ref))
    G = rng.standard_normal(ref.shape).astype(np.float32)
    gx, gb = torch.autograd.grad(out, (Xt, Bt), _t(G, cuda))
    acc = np.zeros((N, 128))
    np.add.at(acc, snd, G[:, :128].astype(np.float64))
    np.add.at(acc, rcv, G[:, 128:256].astype(np.float64))
    np.testing.assert_allclose(gx.cpu().numpy(), acc, rtol=1e-5, atol=1e-4)
    assert torch.equal(gb.cpu(), torch.from_numpy(G[:, 256:]))


def test_gather_cat_unaligned_rows_and_strided_views(cuda):
    from fastmd_b200 import ops

    rng = np.random.default_rng(4)
    packed = _t(rng.standard_normal((50, 21)).astype(np.float32), cuda)
    view = packed[:, 7:14]  # row stride 21, width 7: the scalar path
    idx = _t(rng.integers(0, 50, 33), cuda)
    out = ops.gather_cat([(view, idx), (view[:33], None)])
    ref = np.concatenate([packed.cpu().numpy()[:, 7:14][idx.cpu().numpy()], packed.cpu().numpy()[:33, 7:14]], 1)
    assert torch.equal(out.cpu(), torch.from_numpy(ref))


def test_gather_cat_empty_and_out_of_range_flag(cuda):
    from fastmd_b200 import ops

    X = torch.randn(5, 8, device=cuda)
    empty = torch.zeros(0, dtype=torch.int64, device=cuda)
    assert ops.aligned_gather_cat3(torch.zeros(0, 8, device=cuda), X, empty, empty).shape == (0, 24)
    ops.read_flags(cuda)
    bad = torch.tensor([0, 7, -1], device=cuda)
    out = ops.aligned_gather_cat3(torch.ones(3, 8, device=cuda), X, bad, bad)
    assert ops.read_flags(cuda) & 1
    assert torch.equal(out[1, 8:], torch.zeros(16, device=cuda))  # skipped, zero-filled
    assert torch.equal(out[0, 8:16], X[0])


@pytest.mark.parametrize("tag", ["identity", "perm_weighted", "wide_skip", "narrow"])
def test_csr_segment_sum_matches_reference(cuda, tag):
    from fastmd_b200 import ops

    g = golden("segment_sum")
    S, identity, weighted, skip = (int(v) for v in g[f"segsum_{tag}_meta"])
    seg, perm, off, V, W, G = (_t(g[f"segsum_{tag}_{k}"], cuda) for k in ("seg", "perm", "off", "V", "W", "G"))
    V.requires_grad_(True)
    W.requires_grad_(bool(weighted))
    kw = dict(weight=W if weighted else None, skip_segment=skip)
    if identity:
        out = ops.csr_segment_sum(V, seg, S, None, ops.csr_offsets(seg, S), True, **kw)
    else:
        out = ops.csr_segment_sum(V, seg, S, **kw)  # CSR built on the device
    np.testing.assert_allclose(out.detach().cpu().numpy(), g[f"segsum_{tag}_out"], rtol=1e-5, atol=2e-5)
    inputs = (V, W) if weighted else (V,)
    grads = torch.autograd.grad(out, inputs, G)
    assert torch.equal(grads[0].cpu(), torch.from_numpy(g[f"segsum_{tag}_gvalue"]))
    if weighted:
        assert torch.equal(grads[1].cpu(), torch.from_numpy(g[f"segsum_{tag}_gweight"]))
    again = ops.csr_segment_sum(V, seg, S, **kw) if not identity else \
        ops.csr_segment_sum(V, seg, S, None, ops.csr_offsets(seg, S), True, **kw)
    assert torch.equal(out, again)  # deterministic


def test_csr_metadata_is_a_stable_sort(cuda):
    from fastmd_b200 import ops

    rng = np.random.default_rng(5)
    for rows, S in ((0, 4), (1, 1), (1000, 7), (70000, 1531)):
        seg = rng.integers(0, S, rows)
        perm, off = ops.segment_csr(_t(seg, cuda), S)
        p, o = oops.segment_csr(seg, S)
        assert np.array_equal(perm.cpu().numpy(), p) and np.array_equal(off.cpu().numpy(), o)
        srt = np.sort(seg)
        assert np.array_equal(ops.csr_offsets(_t(srt, cuda), S).cpu().numpy(), o)


def test_segment_count_and_aggregate(cuda):
    from fastmd_b200 import ops

    rng = np.random.default_rng(6)
    seg = rng.integers(0, 9, 500)
    data = rng.standard_normal((500, 12)).astype(np.float32)
    counts = ops.segment_count(_t(seg, cuda), 11).cpu().numpy()
    assert np.array_equal(counts, np.bincount(seg, minlength=11))
    mean = ops.aggregate(_t(data, cuda), _t(seg, cuda), num_segment=11).cpu().numpy()
    ref = oops.segment_sum(data, seg, 11) / np.maximum(np.bincount(seg, minlength=11), 1)[:, None]
    np.testing.assert_allclose(mean, ref, rtol=1e-5, atol=1e-6)


def test_large_segment_sum_against_oracle(cuda):
    """The op-microbenchmark shape, scaled: 54 receivers-sorted rows per node, width 256."""
    from fastmd_b200 import ops

    rng = np.random.default_rng(7)
    N, D = 2000, 256
    seg = np.sort(rng.integers(0, N, 54 * N))
    V = rng.standard_normal((seg.size, D)).astype(np.float32)
    segt = _t(seg, cuda)
    out = ops.csr_segment_sum(_t(V, cuda), segt, N, None, ops.csr_offsets(segt, N), True)
    ref = oops.segment_sum(V, seg, N)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=5e-5)


def test_gather_rows_bwd_long_runs(cuda):
    """fmd_gather_rows_bwd_long (eight warps per source row, for runs of tens to hundreds of rows) against
    float64 row sums and against fmd_gather_rows_bwd, on sorted (identity) and permuted CSRs."""
    from fastmd_b200._lib import call, ptr, stream
    from fastmd_b200.ops import segment_csr

    gen = np.random.default_rng(5)
    rows, n_src, width = 17_850, 135, 256
    for sorted_index in (True, False):
        seg = gen.integers(0, n_src, rows)
        if sorted_index:
            seg = np.sort(seg)
        idx = torch.from_numpy(seg.astype(np.int64)).to(cuda)
        perm, off = segment_csr(idx, n_src)
        gout = torch.from_numpy(gen.standard_normal((rows, width)).astype(np.float32)).to(cuda)
        out = {}
        for name in ("fmd_gather_rows_bwd_long", "fmd_gather_rows_bwd"):
            grad = torch.full((n_src, width), float("nan"), device=cuda)
            call(name, ptr(gout), width, 0, width, ptr(perm), ptr(off), n_src, ptr(grad), width, 0, stream(cuda))
            out[name] = grad.cpu().numpy()
        ref = np.zeros((n_src, width))
        np.add.at(ref, seg, gout.cpu().numpy().astype(np.float64))
        for grad in out.values():
            assert np.abs(grad - ref).max() <= 2e-5 * np.abs(ref).max()
