"""FP64 restatement of the NequIP-architecture (SevenNet-0-style) potential -- TEST INFRASTRUCTURE ONLY.

**parity unpinned**: the reference runs SevenNet through ``sevenn==0.13.0`` (fastmd/models/sevennet.py),
which is not vendored and not installed here; this restates the published NequIP/SevenNet equations
(an E(3)-equivariant interatomic potential: species embedding, interaction blocks of a
self-connection, a linear, a radial-weighted tensor-product convolution over the neighbours, a second
linear and a gated nonlinearity, then a scalar readout; forces are minus the position gradient)
with the architecture of BASELINE config 3: irreps 128x0e + 64x1e + 32x2e (no parity), spherical
harmonics up to l = 2 ("component" normalisation), 8 Bessel radial functions with a polynomial
envelope (p = 6), cutoff 5 A, 5 interaction blocks, radial network 8 -> 64 -> 64 -> weights (SiLU,
no bias), average neighbour count normalisation, readout 128 -> 64 -> 1.

The Clebsch-Gordan tensors of the real basis are derived numerically here (the equivariant map
between the representations, from random rotations; unique up to sign and scale, fixed as the
unit-Frobenius-times-sqrt(2 l3 + 1) tensor with a positive largest entry), the same derivation the
product uses, so both sides share the coupling constants to ~1e-15.
"""
from __future__ import annotations

import numpy as np
import torch

MULT = (128, 64, 32)
DIM = (1, 3, 5)
PATHS = [(l1, l2, l3) for l1 in range(3) for l2 in range(3) for l3 in range(3) if abs(l1 - l2) <= l3 <= l1 + l2]


def sh(u):
    """Real spherical harmonics l = 0, 1, 2 of unit vectors [..., 3] (component normalisation):
    [1 | sqrt3 (x, y, z) | sqrt15 xy, sqrt15 yz, sqrt5/2 (3z^2 - 1), sqrt15 xz, sqrt15/2 (x^2 - y^2)]."""
    x, y, z = u[..., 0], u[..., 1], u[..., 2]
    s3, s5, s15 = 3.0 ** 0.5, 5.0 ** 0.5, 15.0 ** 0.5
    one = torch.ones_like(x) if torch.is_tensor(x) else np.ones_like(x)
    stack = torch.stack if torch.is_tensor(x) else np.stack
    return stack([one, s3 * x, s3 * y, s3 * z, s15 * x * y, s15 * y * z, s5 / 2 * (3 * z * z - 1), s15 * x * z,
                  s15 / 2 * (x * x - y * y)], -1)


def _sh_l(l, u):
    return sh(u)[..., [0] if l == 0 else ([1, 2, 3] if l == 1 else [4, 5, 6, 7, 8])]


def clebsch_gordan(l1, l2, l3, seed=0):
    """[2 l3 + 1, 2 l1 + 1, 2 l2 + 1] float64 coupling tensor of the real basis of ``sh``."""
    rng = np.random.default_rng(seed)

    def rot():
        q = rng.normal(size=4)
        a, b, c, d = q / np.linalg.norm(q)
        return np.array([[a * a + b * b - c * c - d * d, 2 * (b * c - a * d), 2 * (b * d + a * c)],
                         [2 * (b * c + a * d), a * a - b * b + c * c - d * d, 2 * (c * d - a * b)],
                         [2 * (b * d - a * c), 2 * (c * d + a * b), a * a - b * b - c * c + d * d]])

    def wigner(l, R):
        pts = rng.normal(size=(64, 3))
        pts /= np.linalg.norm(pts, axis=1, keepdims=True)
        dt, *_ = np.linalg.lstsq(_sh_l(l, pts), _sh_l(l, pts @ R.T), rcond=None)
        return dt.T

    n1, n2, n3 = 2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1
    rows = []
    for _ in range(4):
        R = rot()
        k = np.kron(wigner(l1, R), wigner(l2, R))
        rows.append(np.kron(np.eye(n1 * n2), wigner(l3, R)) - np.kron(k.T, np.eye(n3)))
    _, _, vt = np.linalg.svd(np.vstack(rows))
    c = vt[-1].reshape(n1 * n2, n3).T
    c = c / np.linalg.norm(c) * np.sqrt(n3)
    c = c * np.sign(c.flat[np.argmax(np.abs(c))])
    c[np.abs(c) < 1e-12] = 0.0
    return c.reshape(n3, n1, n2)


def radial_basis(d, r_max, n_basis=8, p=6):
    """Bessel functions sqrt(2/rc) sin(n pi d / rc) / d times the polynomial envelope of order p."""
    x = d / r_max
    env = (1.0 - (p + 1) * (p + 2) / 2 * x ** p + p * (p + 2) * x ** (p + 1) - p * (p + 1) / 2 * x ** (p + 2))
    env = torch.where(x < 1.0, env, torch.zeros_like(env))
    n = torch.arange(1, n_basis + 1, dtype=d.dtype)
    return (2.0 / r_max) ** 0.5 * torch.sin(n * np.pi * d[:, None] / r_max) / d[:, None] * env[:, None]


def _split(x):
    """[N, 480] -> [x0 [N,128,1], x1 [N,64,3], x2 [N,32,5]]."""
    out, off = [], 0
    for m, d in zip(MULT, DIM):
        out.append(x[:, off:off + m * d].reshape(-1, m, d))
        off += m * d
    return out


def energy_forces(weights, config, positions, cell, numbers, center, neighbor, images):
    """(energy (float), forces [N, 3]) in float64; ``weights`` the numpy arrays of the model's
    ``init_weights`` (element rows indexed by atomic number - 1), edges (centre i receives from
    neighbour j, image of j)."""
    t = lambda a: torch.as_tensor(np.asarray(a), dtype=torch.float64)  # noqa: E731
    pos = t(positions).requires_grad_(True)
    cellt = t(cell)
    ci, nj = torch.as_tensor(center, dtype=torch.long), torch.as_tensor(neighbor, dtype=torch.long)
    vec = pos[nj] - pos[ci] + t(images) @ cellt
    d = vec.norm(dim=1)
    Y = sh(vec / d[:, None])
    B = radial_basis(d, config.r_max, config.num_bessel, config.poly_p)
    N = pos.shape[0]
    elem = torch.as_tensor(np.asarray(numbers), dtype=torch.long) - 1  # atomic number -> element row
    cg = {p: t(clebsch_gordan(*p)) for p in PATHS}
    x = torch.zeros(N, 480, dtype=torch.float64)
    x[:, :128] = t(weights["embed"])[elem]
    for L in range(config.num_layers):
        W = {k: t(v) for k, v in weights.items() if k.startswith(f"L{L}.")}
        xs = _split(x)
        # self-connection: an element-dependent linear per l
        sc = [torch.einsum("nud,nuv->nvd", xs[l], W[f"L{L}.sc{l}"][elem]) for l in range(3)]
        # first linear per l
        h = [torch.einsum("nud,uv->nvd", xs[l], W[f"L{L}.lin1_{l}"]) for l in range(3)]
        # radial weights per edge
        r1 = torch.nn.functional.silu(B @ W[f"L{L}.rad1"].T)
        r2 = torch.nn.functional.silu(r1 @ W[f"L{L}.rad2"].T)
        wts = r2 @ W[f"L{L}.rad3"].T  # [E, 960]
        msgs = {0: [], 1: [], 2: []}
        woff = 0
        for (l1, l2, l3) in PATHS:
            u = MULT[l1]
            w = wts[:, woff:woff + u]
            woff += u
            yl2 = Y[:, [0] if l2 == 0 else ([1, 2, 3] if l2 == 1 else [4, 5, 6, 7, 8])]
            m = torch.einsum("kij,eui,ej->euk", cg[(l1, l2, l3)], h[l1][nj], yl2) * w[:, :, None]
            agg = torch.zeros(N, u, 2 * l3 + 1, dtype=torch.float64).index_add_(0, ci, m)
            msgs[l3].append(agg / config.avg_num_neighbors)
        mcat = [torch.cat(msgs[l], 1) for l in range(3)]  # [N, 224, 1], [N, 384, 3], [N, 352, 5]
        o = [torch.einsum("nud,uv->nvd", mcat[l], W[f"L{L}.lin2_{l}"]) for l in range(3)]
        scal = torch.nn.functional.silu(o[0][:, :128, 0])
        gates = torch.sigmoid(o[0][:, 128:, 0])
        g1 = o[1] * gates[:, :64, None]
        g2 = o[2] * gates[:, 64:, None]
        x = torch.cat([(scal + sc[0][:, :, 0]), (g1 + sc[1]).reshape(N, -1), (g2 + sc[2]).reshape(N, -1)], 1)
    hid = x[:, :128] @ t(weights["readout1"]).T
    e_atom = (hid @ t(weights["readout2"]).T)[:, 0] * config.scale + config.shift
    energy = e_atom.sum()
    (grad,) = torch.autograd.grad(energy, pos)
    return float(energy.detach()), (-grad).detach().numpy()
