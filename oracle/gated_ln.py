"""CPU restatement of the reference's fused GatedMLP epilogue -- TEST INFRASTRUCTURE ONLY.

fastmd/models/matris/op/triton_gated_ln.py (``_gated_ln_fwd`` :57 / ``_gated_ln_fwd_2d`` :205 and their
backwards :127 / :280), per row of width D in FP32:

    x_c = core_x (+ core_lb),  mu = sum(x_c) / D,  rs = 1 / sqrt(sum((x_c - mu)^2) / D + eps)
    y_c = (x_c - mu) rs w_c + b_c,   core = y_c sigmoid(y_c),   gate = sigmoid(y_g) (same for the gate)
    out = core * gate (+ residual * res_weight)

and the backward from the saved mean / rstd: ``d_core_y = g gate s (1 + y (1 - s))``,
``d_gate_y = g core gate (1 - gate)``, ``dx = (dxhat - mean(dxhat) - xhat mean(dxhat xhat)) rs`` with
``dxhat = dy w``. Pinned against the reference's 2-D kernels under TRITON_INTERPRET=1
(tests/golden/gated_ln.npz) to FP32 rounding (the row sums are taken in another order).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _sig(x):
    return F32(1) / (F32(1) + np.exp(-x))


def _ln(x, w, b, eps, D):
    mu = (x.sum(axis=1, dtype=F32) / F32(D)).astype(F32)
    c = x - mu[:, None]
    rs = (F32(1) / np.sqrt((c * c).sum(axis=1, dtype=F32) / F32(D) + F32(eps))).astype(F32)
    return c * rs[:, None] * w[None, :] + b[None, :], mu, rs


def forward(core_x, gate_x, cw, cb, gw, gb, eps_core=1e-5, eps_gate=1e-5, core_lb=None, gate_lb=None, residual=None,
            res_weight=None):
    """(out, core_mean, core_rstd, gate_mean, gate_rstd)."""
    cx, gx = np.asarray(core_x, F32), np.asarray(gate_x, F32)
    if core_lb is not None:
        cx, gx = cx + np.asarray(core_lb, F32)[None, :], gx + np.asarray(gate_lb, F32)[None, :]
    D = cx.shape[1]
    cy, cmu, crs = _ln(cx, np.asarray(cw, F32), np.asarray(cb, F32), eps_core, D)
    gy, gmu, grs = _ln(gx, np.asarray(gw, F32), np.asarray(gb, F32), eps_gate, D)
    out = (cy * _sig(cy)) * _sig(gy)
    if residual is not None:
        out = out + np.asarray(residual, F32) * np.asarray(res_weight, F32)[None, :]
    return out.astype(F32), cmu, crs, gmu, grs


def backward(core_x, gate_x, cw, cb, gw, gb, grad, cmu, crs, gmu, grs, core_lb=None, gate_lb=None, res_weight=None):
    """(grad_core_x, grad_gate_x, grad_residual or None)."""
    cx, gx = np.asarray(core_x, F32), np.asarray(gate_x, F32)
    if core_lb is not None:
        cx, gx = cx + np.asarray(core_lb, F32)[None, :], gx + np.asarray(gate_lb, F32)[None, :]
    D = cx.shape[1]
    g = np.asarray(grad, F32)
    cxh = (cx - cmu[:, None]) * crs[:, None]
    cy = cxh * cw[None, :] + cb[None, :]
    cs = _sig(cy)
    core = cy * cs
    gxh = (gx - gmu[:, None]) * grs[:, None]
    gy = gxh * gw[None, :] + gb[None, :]
    gate = _sig(gy)
    d_cy = g * gate * (cs * (F32(1) + cy * (F32(1) - cs)))
    d_gy = g * core * (gate * (F32(1) - gate))

    def ln_bwd(dy, w, xh, rs):
        dxh = dy * w[None, :]
        m1 = dxh.sum(axis=1, dtype=F32) / F32(D)
        m2 = (dxh * xh).sum(axis=1, dtype=F32) / F32(D)
        return ((dxh - m1[:, None] - xh * m2[:, None]) * rs[:, None]).astype(F32)

    gres = (g * np.asarray(res_weight, F32)[None, :]).astype(F32) if res_weight is not None else None
    return ln_bwd(d_cy, cw, cxh, crs), ln_bwd(d_gy, gw, gxh, grs), gres
