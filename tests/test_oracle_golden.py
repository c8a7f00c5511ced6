"""The CPU oracle against the golden vectors of the reference's own code (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from conftest import golden
from oracle import neighbors as onb
from oracle import nhc as onhc
from oracle import ops as oops


def test_gather_cat3_matches_reference_kernels():
    g = golden("gather_cat")
    for tag in ("small", "wide", "odd"):
        A, X, ia, ib, G = (g[f"cat3_{tag}_{k}"] for k in ("A", "X", "ia", "ib", "G"))
        np.testing.assert_array_equal(oops.aligned_gather_cat3(A, X, ia, ib), g[f"cat3_{tag}_out"])
        ga, gx = oops.aligned_gather_cat3_bwd(G, X.shape[0], ia, ib)
        np.testing.assert_array_equal(ga, g[f"cat3_{tag}_grad_aligned"])
        # the reference scatters with float32 atomics: equal up to the summation order
        np.testing.assert_allclose(gx, g[f"cat3_{tag}_grad_gathered"], rtol=1e-5, atol=1e-5)


def test_gather_cat4_matches_reference_kernels():
    g = golden("gather_cat")
    out = oops.aligned_gather_cat4(g["cat4_A"], g["cat4_Xa"], g["cat4_ia"], g["cat4_Xb"], g["cat4_ib"], g["cat4_ic"])
    np.testing.assert_array_equal(out, g["cat4_out"])
    ga, g1, g2 = oops.aligned_gather_cat4_bwd(g["cat4_G"], g["cat4_Xa"].shape[0], g["cat4_Xb"].shape[0],
                                              g["cat4_ia"], g["cat4_ib"], g["cat4_ic"])
    np.testing.assert_array_equal(ga, g["cat4_grad_aligned"])
    np.testing.assert_allclose(g1, g["cat4_grad_a"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(g2, g["cat4_grad_b"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tag", ["identity", "perm_weighted", "wide_skip", "narrow"])
def test_csr_segment_sum_matches_reference_kernels(tag):
    g = golden("segment_sum")
    S, identity, weighted, skip = (int(v) for v in g[f"segsum_{tag}_meta"])
    seg, V, W, G = (g[f"segsum_{tag}_{k}"] for k in ("seg", "V", "W", "G"))
    perm, off = oops.segment_csr(seg, S)
    np.testing.assert_array_equal(perm, g[f"segsum_{tag}_perm"])
    np.testing.assert_array_equal(off, g[f"segsum_{tag}_off"])
    w = W if weighted else None
    out = oops.csr_segment_sum(V, S, None if identity else perm, off, weight=w, skip_segment=skip)
    np.testing.assert_allclose(out, g[f"segsum_{tag}_out"], rtol=1e-5, atol=2e-5)
    gv, gw = oops.csr_segment_sum_bwd(G, V, seg, weight=w, skip_segment=skip)
    np.testing.assert_array_equal(gv, g[f"segsum_{tag}_gvalue"])  # one multiply: exact
    if weighted:
        np.testing.assert_array_equal(gw, g[f"segsum_{tag}_gweight"])


def test_maxwell_boltzmann_bitwise():
    g = golden("nhc")
    np.testing.assert_array_equal(onhc.maxwell_boltzmann_momenta(g["mb_masses"], 500.0, seed=0),
                                  g["mb_momenta_500K_seed0"])


@pytest.mark.parametrize("tag", ["f64_m3_l1", "f32_m3_l1", "f64_m1_l1", "f64_m5_l2"])
def test_nhc_oracle_matches_reference_torch_backend(tag):
    g = golden("nhc")
    n, tchain, tloop, f32, steps = (int(v) for v in g[f"nhc_{tag}_meta"])
    T, dt, tdamp, k = g["nhc_params"]
    q0 = g["nhc_q0"]
    init = g[f"nhc_{tag}_init"]
    masses, q, p = init[:n], init[n:4 * n].reshape(n, 3), init[4 * n:].reshape(n, 3)
    fdt = np.float32 if f32 else np.float64

    def forces(x):
        f = -k * (x - q0)
        return f.astype(fdt), 0.5 * k * float(np.sum((x - q0) ** 2))

    f, e = forces(q)
    nhc = onhc.NHC(masses, q, p, f, temperature_K=T, timestep=dt, tdamp=tdamp, tchain=tchain, tloop=tloop,
                   f32_kick=bool(f32), energy=e)
    flats = [nhc.flat()]
    for _ in range(steps):
        x = nhc.pre_force()
        f, e = forces(x)
        nhc.post_force(f, e)
        flats.append(nhc.flat())
    ref = g[f"nhc_{tag}_flat"]
    mine = np.array(flats)
    assert mine.shape == ref.shape
    scale = np.maximum(np.abs(ref), 1e-300)
    rel = np.max(np.abs(mine - ref) / np.maximum(scale, np.abs(ref).max(axis=0, keepdims=True) * 1e-3 + 1e-30))
    assert rel < 1e-12, rel


@pytest.mark.parametrize("tag", ["perov", "tric"])
def test_refilter_oracle_matches_reference_kernels(tag):
    g = golden("neighbors")
    rc, _ = g[f"nbr_{tag}_cutoffs"]
    wrapped = g[f"nbr_{tag}_wrapped"]
    cell = g[f"nbr_{tag}_cell"]
    # the wrap prologue in the reference's arithmetic (torch small_matmul on CPU)
    w, wraps, _ = onb.wrap(g[f"nbr_{tag}_positions"], cell,
                           inv_cell=np.linalg.inv(cell.astype(np.float32)).astype(np.float32))
    np.testing.assert_array_equal(wraps, g[f"nbr_{tag}_wraps"])
    c, n, img, dist = onb.refilter(wrapped, cell, g[f"nbr_{tag}_cand_matrix"], g[f"nbr_{tag}_cand_shifts"],
                                   g[f"nbr_{tag}_cand_count"], rc)
    c, n, img, dist = onb.canonical(c, n, img, wrapped.shape[0], dist)
    np.testing.assert_array_equal(np.stack([c, n], 1), g[f"nbr_{tag}_edges"])
    np.testing.assert_array_equal(img, g[f"nbr_{tag}_images"])
    np.testing.assert_array_equal(dist, g[f"nbr_{tag}_dist"])


@pytest.mark.parametrize("tag", ["perov", "tric"])
def test_refilter_equals_dense_fp64_search_up_to_ties(tag):
    g = golden("neighbors")
    rc, _ = g[f"nbr_{tag}_cutoffs"]
    wrapped = g[f"nbr_{tag}_wrapped"]
    cell = g[f"nbr_{tag}_cell"]
    dense = onb.dense_pairs(wrapped, cell, rc + 1e-3)
    mine = {(int(a), int(b), *map(int, i)) for (a, b), i in zip(g[f"nbr_{tag}_edges"], g[f"nbr_{tag}_images"])}
    theirs = {key for key, d in dense.items() if d < rc}
    for key in mine ^ theirs:
        assert abs(dense[key] - rc) < 1e-5, key


@pytest.mark.parametrize("tag", ["mace", "matris"])
def test_radial_basis_oracle_matches_reference_module(tag):
    import torch

    from oracle import mace as omace

    g = golden("radial")
    n, rc, p = g[f"radial_{tag}_params"]
    d = torch.as_tensor(g["radial_d"], dtype=torch.float64)
    mine = omace.bessel_envelope(d, float(rc), int(n), float(p)).numpy()
    np.testing.assert_allclose(mine, g[f"radial_{tag}"], rtol=2e-5, atol=2e-6)


def test_neighbor_oracle_candidates_cover_the_dense_search():
    g = golden("neighbors")
    wrapped, cell = g["nbr_perov_wrapped"], g["nbr_perov_cell"]
    nm, ns, nn = onb.candidates(wrapped, cell, 8.0)
    assert int(nn.sum()) == int(g["nbr_perov_cand_count"].sum())
    assert onb.estimate_max_neighbors(8.0, 0.35, 2.0) == 1504
