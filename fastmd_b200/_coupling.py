"""Clebsch-Gordan coupling tensors of the real spherical harmonics up to l = 2 (the NequIP convolution's
constants), derived numerically: the coupling l1 (x) l2 -> l3 is the (one-dimensional) space of maps C
with D_l3(R) C = C (D_l1(R) (x) D_l2(R)) for every rotation R, where D_l(R) is the action of R on the
harmonics (Y_l(R u) = D_l(R) Y_l(u)), fitted by least squares on sample directions; the null space of
the equations of four random rotations, normalised to Frobenius norm sqrt(2 l3 + 1) with a positive
largest entry. Seeded: the same constants on every call."""
from __future__ import annotations

import numpy as np


def _harmonics(l: int, u: np.ndarray) -> np.ndarray:
    x, y, z = u[..., 0], u[..., 1], u[..., 2]
    if l == 0:
        return np.ones(u.shape[:-1] + (1,))
    if l == 1:
        return np.sqrt(3.0) * np.stack([x, y, z], -1)
    s5, s15 = np.sqrt(5.0), np.sqrt(15.0)
    return np.stack([s15 * x * y, s15 * y * z, s5 / 2 * (3 * z * z - 1), s15 * x * z, s15 / 2 * (x * x - y * y)], -1)


def clebsch_gordan(l1: int, l2: int, l3: int, seed: int = 0) -> np.ndarray:
    """[2 l3 + 1, 2 l1 + 1, 2 l2 + 1] float64."""
    rng = np.random.default_rng(seed)

    def rotation():
        a, b, c, d = (q := rng.normal(size=4)) / np.linalg.norm(q)
        return np.array([[a * a + b * b - c * c - d * d, 2 * (b * c - a * d), 2 * (b * d + a * c)],
                         [2 * (b * c + a * d), a * a - b * b + c * c - d * d, 2 * (c * d - a * b)],
                         [2 * (b * d - a * c), 2 * (c * d + a * b), a * a - b * b - c * c + d * d]])

    def action(l, R):
        pts = rng.normal(size=(64, 3))
        pts /= np.linalg.norm(pts, axis=1, keepdims=True)
        dt, *_ = np.linalg.lstsq(_harmonics(l, pts), _harmonics(l, pts @ R.T), rcond=None)
        return dt.T

    n1, n2, n3 = 2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1
    rows = []
    for _ in range(4):
        R = rotation()
        k = np.kron(action(l1, R), action(l2, R))
        rows.append(np.kron(np.eye(n1 * n2), action(l3, R)) - np.kron(k.T, np.eye(n3)))
    _, _, vt = np.linalg.svd(np.vstack(rows))
    c = vt[-1].reshape(n1 * n2, n3).T
    c = c / np.linalg.norm(c) * np.sqrt(n3)
    c = c * np.sign(c.flat[np.argmax(np.abs(c))])
    c[np.abs(c) < 1e-12] = 0.0
    return c.reshape(n3, n1, n2)
