"""Clebsch-Gordan coefficients from Racah's closed formula, in the real basis -- TEST INFRASTRUCTURE ONLY.

The NequIP convolution's coupling constants (fastmd_b200/_coupling.py) are derived numerically from the
equivariance condition. This module derives the same tensors independently, from the published
closed form of the complex (Condon-Shortley) coefficients <l1 m1 l2 m2 | L M> (Racah, Phys. Rev. 62, 438
(1942), eq. 16.6 of the usual tables), moved into the real basis of ``_coupling._harmonics``: with the
real harmonics y_r = U y_c (U fitted from the two sets of functions on sample directions, SciPy's
``sph_harm_y`` for the complex ones), C_real = U_L C (U_l1 (x) U_l2)^-1, made real by its overall phase
and normalised like the product (Frobenius norm sqrt(2L + 1), positive largest entry)."""
from __future__ import annotations

from math import factorial, sqrt

import numpy as np


def racah(l1: int, m1: int, l2: int, m2: int, L: int, M: int) -> float:
    """<l1 m1 l2 m2 | L M> (integer angular momenta)."""
    if M != m1 + m2 or not abs(l1 - l2) <= L <= l1 + l2 or abs(m1) > l1 or abs(m2) > l2 or abs(M) > L:
        return 0.0
    f = factorial
    pre = sqrt((2 * L + 1) * f(L + l1 - l2) * f(L - l1 + l2) * f(l1 + l2 - L) / f(l1 + l2 + L + 1))
    pre *= sqrt(f(L + M) * f(L - M) * f(l1 - m1) * f(l1 + m1) * f(l2 - m2) * f(l2 + m2))
    total = 0.0
    for k in range(0, l1 + l2 - L + 1):
        den = [k, l1 + l2 - L - k, l1 - m1 - k, l2 + m2 - k, L - l2 + m1 + k, L - l1 - m2 + k]
        if min(den) < 0:
            continue
        term = 1.0
        for d in den:
            term *= f(d)
        total += (-1) ** k / term
    return pre * total


def _real_from_complex(l: int, harmonics) -> np.ndarray:
    """U with real(u) = U complex(u) for the real harmonics ``harmonics(l, u)`` of one degree."""
    from scipy.special import sph_harm_y

    rng = np.random.default_rng(7)
    u = rng.normal(size=(200, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    theta, phi = np.arccos(np.clip(u[:, 2], -1, 1)), np.arctan2(u[:, 1], u[:, 0])
    yc = np.stack([sph_harm_y(l, m, theta, phi) for m in range(-l, l + 1)], -1)  # [200, 2l+1]
    yr = harmonics(l, u).astype(complex)
    ut, *_ = np.linalg.lstsq(yc, yr, rcond=None)
    return ut.T


def real_clebsch_gordan(l1: int, l2: int, L: int, harmonics) -> np.ndarray:
    """[2L + 1, 2l1 + 1, 2l2 + 1] float64 in the basis of ``harmonics``, normalised as the product's."""
    cc = np.zeros((2 * L + 1, (2 * l1 + 1) * (2 * l2 + 1)), dtype=complex)
    for a, m1 in enumerate(range(-l1, l1 + 1)):
        for b, m2 in enumerate(range(-l2, l2 + 1)):
            M = m1 + m2
            if abs(M) <= L:
                cc[M + L, a * (2 * l2 + 1) + b] = racah(l1, m1, l2, m2, L, M)
    u1, u2, u3 = (_real_from_complex(l, harmonics) for l in (l1, l2, L))
    cr = u3 @ cc @ np.linalg.inv(np.kron(u1, u2))
    cr = cr / (cr.flat[np.argmax(np.abs(cr))] / abs(cr.flat[np.argmax(np.abs(cr))]))  # the overall phase
    c = cr.real / np.linalg.norm(cr.real) * np.sqrt(2 * L + 1)
    c = c * np.sign(c.flat[np.argmax(np.abs(c))])
    assert np.abs(cr.imag).max() < 1e-9 * np.abs(cr.real).max()
    return c.reshape(2 * L + 1, 2 * l1 + 1, 2 * l2 + 1)
