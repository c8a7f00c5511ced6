"""Cell-list candidates, the per-step re-filter and the ragged list on the GPU against the oracle
(whose restatement of the reference's re-filter is pinned bitwise to the reference's kernels)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import neighbors as onb

pytestmark = pytest.mark.gpu


def _perov(seed=0):
    from fastmd_b200.structures import perovskite

    return perovskite(seed=seed)


def _builder(cell, numbers, u_capacity, cuda, skin=2.0, replicas=1, rc=6.0, **kw):
    from fastmd_b200.graph import FixedCapacityGraphBuilder

    return FixedCapacityGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32), atomic_numbers=torch.tensor(numbers),
                                     u_capacity=u_capacity, atom_graph_cutoff=rc, candidate_cutoff=rc + skin,
                                     device=cuda, replicas=replicas, **kw)


def _edges_of(builder):
    n = int(builder.batch.n_edges.item())
    ei = builder.batch.edge_index[:n].cpu().numpy().astype(np.int64)
    im = builder.batch.edge_image[:n].cpu().numpy().round().astype(np.int64)
    return n, ei, im


def _oracle_refilter(builder, pos32):
    """The oracle re-filter on the builder's own candidates and wrapped positions."""
    wrapped, _, _ = onb.wrap(pos32, builder.cell.cpu().numpy(), inv_cell=onb.inverse_cell(builder.cell.cpu().numpy()))
    c, nb, im, _ = onb.refilter(wrapped, builder.cell.cpu().numpy(), builder.cand_nbr.cpu().numpy(),
                                builder.cand_shift.cpu().numpy(), builder.cand_count.cpu().numpy(),
                                builder.atom_graph_cutoff, wrap_delta=builder.wrap_delta.cpu().numpy())
    return wrapped, c, nb, im


@pytest.mark.parametrize("tag", ["perov", "tric"])
def test_candidates_match_dense_search_and_are_canonical(cuda, tag):
    g = golden("neighbors")
    cell, pos = g[f"nbr_{tag}_cell"], g[f"nbr_{tag}_positions"]
    b = _builder(cell, np.full(pos.shape[0], 14), 8192, cuda)
    b.refresh_candidates(torch.from_numpy(pos).to(cuda))
    assert int(b.refresh_flags.item()) == 0
    counts = b.cand_count.cpu().numpy()
    nbr, sh = b.cand_nbr.cpu().numpy(), b.cand_shift.cpu().numpy()
    wrapped, _, _ = onb.wrap(pos, cell, inv_cell=onb.inverse_cell(cell))
    dense = onb.dense_pairs(wrapped, cell, b.candidate_cutoff + 1e-3)
    mine = set()
    for i in range(pos.shape[0]):
        row = [(int(nbr[i, k]), *map(int, sh[i, k])) for k in range(counts[i])]
        keys = onb.sort_key(np.full(len(row), i), [r[0] for r in row], np.array([r[1:] for r in row]), pos.shape[0])
        assert np.all(np.diff(keys) > 0)  # canonical, no duplicates
        mine.update((i, *r) for r in row)
    theirs = {k for k, d in dense.items() if d < b.candidate_cutoff}
    for key in mine ^ theirs:
        assert abs(dense[key] - b.candidate_cutoff) < 1e-4, key


@pytest.mark.parametrize("seed", [0, 5])
def test_refilter_bitwise_equals_oracle_and_dense_search(cuda, seed):
    pos, cell, numbers, _ = _perov(seed)
    b = _builder(cell, numbers, 4096, cuda)
    pos32 = pos.astype(np.float32)
    batch, status = b.build(torch.from_numpy(pos32).to(cuda))
    assert int(status.flags.item()) == 0
    n, ei, im = _edges_of(b)
    wrapped, c, nb, oim = _oracle_refilter(b, pos32)
    assert np.array_equal(batch.positions.cpu().numpy(), wrapped)
    c, nb, oim = onb.canonical(c, nb, oim, pos.shape[0])
    assert n == c.size
    assert np.array_equal(ei, np.stack([c, nb], 1)) and np.array_equal(im, oim)
    dense = onb.dense_pairs(wrapped, cell, 6.0 + 1e-3)
    mine = {(int(a), int(x), *map(int, i)) for (a, x), i in zip(ei, im)}
    theirs = {k for k, d in dense.items() if d < 6.0}
    for key in mine ^ theirs:
        assert abs(dense[key] - 6.0) < 1e-5, key
    if seed == 0:
        assert n == 2054


def test_padding_csr_and_capacity(cuda):
    pos, cell, numbers, _ = _perov(0)
    N = pos.shape[0]
    b = _builder(cell, numbers, 1027 + 40, cuda)
    batch, status = b.build(torch.from_numpy(pos).to(cuda))
    n, ei, im = _edges_of(b)
    assert int(status.flags.item()) == 0 and not bool(status.overflow)
    rows = batch.edge_index.cpu().numpy()
    pad = rows[n:]
    assert np.array_equal(pad[:, 0], pad[:, 1])
    assert np.array_equal(pad[:, 0], np.arange(pad.shape[0]) % N)
    shift = batch.edge_image[n:].cpu().numpy() @ cell
    assert np.all(np.linalg.norm(shift, axis=1) >= 12.0)
    off = batch.recv_off.cpu().numpy()
    assert off[0] == 0 and off[-1] == n and np.all(np.diff(off) >= 0)
    assert np.array_equal(np.repeat(np.arange(N), np.diff(off)), ei[:, 0])
    soff, sperm = batch.send_off.cpu().numpy(), batch.send_perm.cpu().numpy()
    assert soff[-1] == n
    for j in range(N):
        run = sperm[soff[j]:soff[j + 1]]
        assert np.all(np.diff(run) > 0) and np.all(ei[run, 1] == j)
    assert sorted(sperm[:n].tolist()) == list(range(n))
    # one pair short: overflow, nothing written past the capacity
    small = _builder(cell, numbers, n // 2 - 1, cuda)
    _, st = small.build(torch.from_numpy(pos).to(cuda))
    assert bool(st.overflow) and int(st.edge_count.item()) == n
    from fastmd_b200.graph import fixed_capacity_exceeded
    assert bool(fixed_capacity_exceeded(st, small))


def test_reused_candidates_equal_a_fresh_build_and_skin_flag(cuda):
    pos, cell, numbers, _ = _perov(0)
    owner = _builder(cell, numbers, 4096, cuda, minimum_image=True)
    fresh = _builder(cell, numbers, 4096, cuda, minimum_image=True)
    base = torch.from_numpy(pos).to(cuda).float()
    owner.refresh_candidates(base)
    gen = torch.Generator(device=cuda).manual_seed(7)
    for step in range(4):
        moved = base + 0.4 * owner.skin * (torch.rand(base.shape, device=cuda, generator=gen) - 0.5)
        moved[step::5] += owner.cell[step % 3] * (1 if step % 2 else -1)  # wrapped by the caller
        _, st = owner.build(moved, rebuild_candidates=False)
        assert int(st.flags.item()) == 0
        fresh.build(moved, rebuild_candidates=True)
        for field in ("edge_index", "edge_image", "positions", "n_edges", "recv_off", "send_off", "send_perm"):
            assert torch.equal(getattr(owner.batch, field), getattr(fresh.batch, field)), field
    jumped = base.clone()
    jumped[0, 0] += 0.6 * owner.skin
    _, st = owner.build(jumped, rebuild_candidates=False)
    assert bool(st.overflow) and not bool(st.candidate_valid)


def test_replica_union_equals_single_systems(cuda):
    R = 3
    systems = [_perov(seed) for seed in range(R)]
    cell, numbers = systems[0][1], systems[0][2]
    N = numbers.size
    union = _builder(cell, numbers, 3 * 4096, cuda, replicas=R)
    pos = np.concatenate([s[0] for s in systems]).astype(np.float32)
    _, st = union.build(torch.from_numpy(pos).to(cuda))
    assert int(st.flags.item()) == 0
    n, ei, im = _edges_of(union)
    start = 0
    for r, s in enumerate(systems):
        single = _builder(cell, numbers, 4096, cuda)
        single.build(torch.from_numpy(s[0].astype(np.float32)).to(cuda))
        m, sei, sim = _edges_of(single)
        assert np.array_equal(ei[start:start + m], sei + r * N) and np.array_equal(im[start:start + m], sim)
        assert np.array_equal(union.batch.positions[r * N:(r + 1) * N].cpu(), single.batch.positions.cpu())
        start += m
    assert start == n


def test_ragged_neighbor_list_equals_oracle(cuda):
    from fastmd_b200.graph import neighbor_list
    from fastmd_b200.structures import random_box

    pos, cell, _ = random_box(3000, density=0.06, seed=2)
    c, nb, im, d, wrapped, off = neighbor_list(torch.from_numpy(pos).float().to(cuda),
                                               torch.from_numpy(cell).float(), 6.0, return_wrapped=True)
    c, nb, im, d = (t.cpu().numpy() for t in (c, nb, im, d))
    w = wrapped.cpu().numpy()
    ow, _, _ = onb.wrap(pos.astype(np.float32), cell.astype(np.float32),
                        inv_cell=onb.inverse_cell(cell.astype(np.float32)))
    assert np.array_equal(w, ow)
    dense = onb.dense_pairs(w, cell, 6.0 + 1e-3)
    keys = np.array(sorted(k for k, dd in dense.items() if dd < 6.0 + 1e-5))
    oc, onb_, oim = keys[:, 0], keys[:, 1], keys[:, 2:]
    keep, odist = onb.ragged_filter(w, cell.astype(np.float32), oc, onb_, oim, 6.0)
    oc, onb_, oim, odist = oc[keep], onb_[keep], oim[keep], odist[keep]
    oc, onb_, oim, odist = onb.canonical(oc, onb_, oim, pos.shape[0], odist)
    assert np.array_equal(c, oc) and np.array_equal(nb, onb_) and np.array_equal(im, oim)
    assert np.array_equal(d, odist)
    assert np.array_equal(off.cpu().numpy(), np.searchsorted(c, np.arange(pos.shape[0] + 1)))


def _candidates_then_eager_filter(pos32, cell32, rc, bmax, cuda):
    """The eager path as the composition the reference runs: this library's cell-list candidates at
    rc + 1e-6 (fmd_candidates_build: the candidate test in the staged float32 arithmetic), then the
    oracle's eager re-filter (gpu_graph_builder.py:186-192) and the canonical order."""
    import ctypes

    from fastmd_b200._lib import call, ptr, stream
    from fastmd_b200.graph import _host_cell

    n = pos32.shape[0]
    _, cell_ptr = _host_cell(torch.from_numpy(cell32))
    cand_cut = float(np.float32(rc) + np.float32(1e-6))
    nbytes = ctypes.c_size_t(0)
    call("fmd_cell_list_workspace_bytes", cell_ptr, cand_cut, n, 1, ctypes.byref(nbytes))
    ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=cuda)
    nbr = torch.empty(n, bmax, dtype=torch.int32, device=cuda)
    shift = torch.empty(n, bmax, 3, dtype=torch.int32, device=cuda)
    count = torch.empty(n, dtype=torch.int32, device=cuda)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    call("fmd_candidates_build", ptr(torch.from_numpy(pos32).to(cuda)), cell_ptr, n, 1, cand_cut, bmax, ptr(nbr),
         ptr(shift), ptr(count), None, None, None, ptr(ws), ws.numel(), ptr(flags), stream(cuda))
    count = count.cpu().numpy()
    assert int(flags.item()) == 0 and count.max() <= bmax
    rows = np.repeat(np.arange(n), count)
    slots = np.concatenate([np.arange(c) for c in count])
    nb, im = nbr.cpu().numpy()[rows, slots].astype(np.int64), shift.cpu().numpy()[rows, slots].astype(np.int64)
    wrapped, _, _ = onb.wrap(pos32, cell32, inv_cell=onb.inverse_cell(cell32))
    keep, dist = onb.ragged_filter(wrapped, cell32, rows, nb, im, rc)
    return onb.canonical(rows[keep], nb[keep], im[keep], n, dist[keep])


def _assert_ragged_equals(pos32, cell32, rc, bmax, cuda, **kw):
    from fastmd_b200.graph import neighbor_list

    oc, onb_, oim, odist = _candidates_then_eager_filter(pos32, cell32, rc, bmax, cuda)
    c, nb, im, d, _, off = neighbor_list(torch.from_numpy(pos32).to(cuda), torch.from_numpy(cell32), rc,
                                         return_wrapped=True, **kw)
    assert np.array_equal(c.cpu().numpy(), oc) and np.array_equal(nb.cpu().numpy(), onb_)
    assert np.array_equal(im.cpu().numpy(), oim) and np.array_equal(d.cpu().numpy(), odist)
    assert np.array_equal(off.cpu().numpy(), np.searchsorted(oc, np.arange(pos32.shape[0] + 1)))
    return odist


def test_ragged_list_at_the_cutoff_equals_candidates_then_the_eager_filter(cuda):
    """A simple cubic lattice of spacing rc / 2 jittered by a few float32 ulps: thousands of pairs lie
    within 1e-5 A of rc, where the candidate test (rc + 1e-6) and the eager distance (< rc) decide
    differently, so the count sweep's shell test runs; bitwise the candidate build followed by the
    eager filter, also when a too small max_neighbors makes the host grow the candidate rows."""
    rng = np.random.default_rng(4)
    g = np.arange(8, dtype=np.float64) * 3.0
    pos = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3) + rng.uniform(-3e-6, 3e-6, (512, 3))
    pos32, cell32 = pos.astype(np.float32), (np.eye(3) * 24.0).astype(np.float32)
    odist = _assert_ragged_equals(pos32, cell32, 6.0, 256, cuda)
    assert int((np.abs(odist - 6.0) < 1e-5).sum()) > 1000
    _assert_ragged_equals(pos32, cell32, 6.0, 256, cuda, max_neighbors=4)


def test_ragged_list_of_dense_neighbourhoods_equals_candidates_then_the_eager_filter(cuda):
    """1,500 atoms at 0.3 / A^3 in a triclinic cell (about 270 neighbours within 6 A, 2 x 2 x 2 cells):
    every neighbourhood stages about 5,000 (atom, image) entries, five chunks of the write sweep."""
    rng = np.random.default_rng(5)
    length = (1500 / 0.3) ** (1.0 / 3.0)
    cell = np.array([[1.0, 0.0, 0.0], [0.3, 1.0, 0.0], [0.2, 0.1, 1.0]]) * length
    pos = rng.uniform(0.0, 1.0, (1500, 3)) @ cell
    _assert_ragged_equals(pos.astype(np.float32), cell.astype(np.float32), 6.0, 600, cuda)


def test_ragged_c2_scale_properties(cuda):
    """The op-microbenchmark system (100k atoms, 0.06 / A^3, rc 6): about 54 neighbours per atom,
    canonical order, and every edge's reverse present (up to float32 ties)."""
    from fastmd_b200.graph import neighbor_list
    from fastmd_b200.structures import random_box

    pos, cell, _ = random_box(100_000, density=0.06, seed=2)
    c, nb, im, d = neighbor_list(torch.from_numpy(pos).float().to(cuda), torch.from_numpy(cell).float(), 6.0)
    E = c.shape[0]
    assert 52.0 < E / 100_000 < 57.0
    key = (c * 100_000 + nb) * 9261 + (im[:, 0] + 10) * 441 + (im[:, 1] + 10) * 21 + im[:, 2] + 10
    assert bool((key[1:] > key[:-1]).all())
    rev = (nb * 100_000 + c) * 9261 + (10 - im[:, 0]) * 441 + (10 - im[:, 1]) * 21 + 10 - im[:, 2]
    found = torch.isin(rev, key)
    missing = (~found).nonzero().flatten()
    assert missing.numel() <= 10 and bool(((d[missing] - 6.0).abs() < 1e-5).all())
    assert float(d.max()) < 6.0


@pytest.mark.parametrize("tag", ["far", "exact_rc"])
def test_padding_rows_equal_the_reference(cuda, tag):
    """The padded rows of a build (2,054 real edges of 2,200 rows) equal the reference's
    ``_pad_self_loops_kernel`` rows; exact-rc padding also publishes the override vector (SevenNet's
    ``PaddingRule("exact_rc_loops")``, sevennet.py:16-22)."""
    from fastmd_b200.graph import PaddingRule

    g = golden("padding")
    total, e_cap, n = (int(v) for v in g[f"pad_{tag}_meta"])
    pos, cell, numbers, _ = _perov(0)
    padding = PaddingRule("exact_rc_loops") if tag == "exact_rc" else None  # pad vector (rc, 0, 0) = (6, 0, 0)
    b = _builder(cell, numbers, e_cap // 2, cuda, padding=padding)
    batch, status = b.build(torch.from_numpy(pos.astype(np.float32)).to(cuda))
    assert int(status.flags.item()) == 0 and int(batch.n_edges.item()) == total
    ei = batch.edge_index.cpu().numpy()
    np.testing.assert_array_equal(ei[total:, 0], g[f"pad_{tag}_center"][total:])
    np.testing.assert_array_equal(ei[total:, 1], g[f"pad_{tag}_neighbor"][total:])
    np.testing.assert_array_equal(batch.edge_image.cpu().numpy()[total:], g[f"pad_{tag}_images"][total:])
    if tag == "exact_rc":
        np.testing.assert_array_equal(batch.edge_vec_override.cpu().numpy(), g["pad_exact_rc_override"])
    else:
        assert batch.edge_vec_override is None


def _refilter_call(name, n_atoms, cuda, cand_count=0):
    """One C-ABI call of the per-step re-filter (``fmd_refilter_edges`` or its allocation-free twin) on
    real device buffers for one system of ``n_atoms`` atoms spread over a 60 A cube: returns the status."""
    import ctypes

    from fastmd_b200._lib import lib, ptr, stream

    bmax, e_cap = 16, 1024
    gen = torch.Generator(device=cuda).manual_seed(5)
    pos = 60.0 * torch.rand((n_atoms, 3), device=cuda, generator=gen)
    i32 = dict(dtype=torch.int32, device=cuda)
    bufs = dict(ref=pos.clone(), wraps=torch.zeros((n_atoms, 3), **i32),
                nbr=torch.full((n_atoms, bmax), n_atoms, **i32), shift=torch.zeros((n_atoms, bmax, 3), **i32),
                count=torch.full((n_atoms,), cand_count, **i32), wrapped=torch.zeros_like(pos),
                wrap_delta=torch.zeros((n_atoms, 3), **i32), edge_index=torch.zeros((e_cap, 2), **i32),
                edge_image=torch.zeros((e_cap, 3), device=cuda), recv_off=torch.zeros(n_atoms + 1, dtype=torch.int64,
                                                                                      device=cuda),
                send_off=torch.zeros(n_atoms + 1, dtype=torch.int64, device=cuda), send_perm=torch.zeros(e_cap, **i32),
                n_edges=torch.zeros(1, dtype=torch.int64, device=cuda), maxd=torch.zeros(1, device=cuda),
                flags=torch.zeros(1, **i32))
    cell = (ctypes.c_float * 9)(60, 0, 0, 0, 60, 0, 0, 0, 60)
    pad = (ctypes.c_int32 * 3)(1, 0, 0)
    b = bufs
    common = [ptr(pos), ctypes.cast(cell, ctypes.c_void_p), n_atoms, 1, ptr(b["ref"]), ptr(b["wraps"]),
              ptr(b["nbr"]), ptr(b["shift"]), ptr(b["count"]), bmax, 6.0, 2.0, e_cap, ctypes.cast(pad, ctypes.c_void_p),
              0, ptr(b["wrapped"]), ptr(b["wrap_delta"]), ptr(b["edge_index"]), ptr(b["edge_image"]),
              ptr(b["recv_off"]), ptr(b["send_off"]), ptr(b["send_perm"]), ptr(b["n_edges"]), ptr(b["maxd"])]
    if name == "fmd_refilter_edges":
        nbytes = ctypes.c_size_t(0)
        assert lib().fmd_refilter_workspace_bytes(n_atoms, 1, ctypes.byref(nbytes)) == 0
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=cuda)
        status = lib().fmd_refilter_edges(*common, ptr(ws), ctypes.c_size_t(ws.numel()), ptr(b["flags"]),
                                          stream(cuda))
    else:
        status = lib().fmd_refilter_edges_noalloc(*common, ptr(b["flags"]), stream(cuda))
    torch.cuda.synchronize()
    if status == 0:
        assert int(b["n_edges"].item()) == 0 and int(b["flags"].item()) == 0  # no candidates: no edges
    return status


@pytest.mark.parametrize("name", ["fmd_refilter_edges", "fmd_refilter_edges_noalloc"])
def test_refilter_per_system_atom_limit(cuda, name):
    """A system's atoms are staged in shared memory (32 bytes each + 4, within 200 KB): 6,399 atoms run,
    6,400 return FMD_ERR_UNSUPPORTED and launch nothing."""
    assert _refilter_call(name, 6399, cuda) == 0
    assert _refilter_call(name, 6400, cuda) == 3  # FMD_ERR_UNSUPPORTED
