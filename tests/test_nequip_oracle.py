"""The NequIP-architecture oracle (parity unpinned: sevenn is absent): the coupling constants are
equivariant, the energy is invariant and the forces covariant under a rotation, and the forces are
minus the energy gradient."""
import numpy as np
import pytest

from oracle import nequip as onq


class _Cfg:
    num_layers, r_max, num_bessel, poly_p, avg_num_neighbors, scale, shift = 2, 5.0, 8, 6, 11.0, 1.0, 0.0


def _weights():
    from fastmd_b200.nequip import NequIPConfig, init_weights

    return init_weights(NequIPConfig(num_layers=2), seed=3)


def _system(seed=0, n=12, box=7.0):
    rng = np.random.default_rng(seed)
    pos = rng.uniform(0, box, (n, 3))
    cell = np.eye(3) * box
    numbers = rng.choice([50, 53, 55], n)
    # all pairs within the cutoff over the images (small box: a few images)
    c, nb, im = [], [], []
    for i in range(n):
        for j in range(n):
            for ix in (-1, 0, 1):
                for iy in (-1, 0, 1):
                    for iz in (-1, 0, 1):
                        if i == j and (ix, iy, iz) == (0, 0, 0):
                            continue
                        d = np.linalg.norm(pos[j] - pos[i] + np.array([ix, iy, iz]) @ cell)
                        if d < 5.0:
                            c.append(i), nb.append(j), im.append((ix, iy, iz))
    return pos, cell, numbers, np.array(c), np.array(nb), np.array(im, float)


@pytest.mark.parametrize("path", [(1, 1, 0), (1, 1, 1), (1, 2, 2), (2, 2, 2), (2, 1, 1)])
def test_couplings_are_equivariant(path):
    rng = np.random.default_rng(1)
    l1, l2, l3 = path
    C = onq.clebsch_gordan(*path)
    u, v = rng.normal(size=3), rng.normal(size=3)
    u, v = u / np.linalg.norm(u), v / np.linalg.norm(v)
    q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
    R = q * np.sign(np.linalg.det(q))
    a = np.einsum("kij,i,j->k", C, onq._sh_l(l1, u), onq._sh_l(l2, v))
    b = np.einsum("kij,i,j->k", C, onq._sh_l(l1, R @ u), onq._sh_l(l2, R @ v))
    # the l3 harmonics of R u transform like the coupled output: compare through a fitted action
    pts = rng.normal(size=(40, 3))
    pts /= np.linalg.norm(pts, axis=1, keepdims=True)
    Dt, *_ = np.linalg.lstsq(onq._sh_l(l3, pts), onq._sh_l(l3, pts @ R.T), rcond=None)
    np.testing.assert_allclose(Dt.T @ a, b, atol=1e-10)


def test_energy_invariant_forces_covariant_and_gradient():
    w = _weights()
    pos, cell, numbers, c, nb, im = _system()
    e, f = onq.energy_forces(w, _Cfg, pos, cell, numbers, c, nb, im)
    q, _ = np.linalg.qr(np.random.default_rng(2).normal(size=(3, 3)))
    R = q * np.sign(np.linalg.det(q))
    e2, f2 = onq.energy_forces(w, _Cfg, pos @ R.T, cell @ R.T, numbers, c, nb, im)
    assert abs(e - e2) < 1e-9 * max(1.0, abs(e))
    np.testing.assert_allclose(f2, f @ R.T, atol=1e-9)
    # finite difference of one coordinate (the edge list is fixed)
    h = 1e-5
    p1, p2 = pos.copy(), pos.copy()
    p1[3, 1] += h
    p2[3, 1] -= h
    ep, _ = onq.energy_forces(w, _Cfg, p1, cell, numbers, c, nb, im)
    em, _ = onq.energy_forces(w, _Cfg, p2, cell, numbers, c, nb, im)
    assert abs(-(ep - em) / (2 * h) - f[3, 1]) < 1e-5 * max(1.0, np.abs(f).max())


def test_coupling_constants_equal_racah_clebsch_gordan():
    """The NequIP coupling constants (derived numerically from equivariance) equal Racah's closed-form
    Clebsch-Gordan coefficients moved into the same real basis, for all 15 paths up to l = 2, up to one
    sign per path (the "positive largest entry" convention is not defined where several entries share the
    largest magnitude; a path's sign is absorbed by its radial weights)."""
    from fastmd_b200._coupling import _harmonics, clebsch_gordan
    from fastmd_b200.nequip import PATHS
    from oracle.clebsch import racah, real_clebsch_gordan

    assert abs(racah(1, 1, 1, -1, 0, 0) - 1 / np.sqrt(3)) < 1e-15  # a textbook entry
    assert abs(racah(1, 1, 1, 0, 2, 1) - 1 / np.sqrt(2)) < 1e-15
    for l1, l2, l3 in PATHS:
        mine = clebsch_gordan(l1, l2, l3)
        ref = real_clebsch_gordan(l1, l2, l3, _harmonics)
        err = min(np.abs(mine - ref).max(), np.abs(mine + ref).max())
        assert err < 1e-9, (l1, l2, l3, err)
