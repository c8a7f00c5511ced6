"""CPU restatement of the reference's segment attention -- TEST INFRASTRUCTURE ONLY.

``out[s, d] = sum_{rows i of segment s} softmax_d(logits[i, d] over the segment) * value[i, d]``
as the reference's CSR kernels compute it in FP32 (fastmd/models/matris/op/triton_segment_attention.py):

* forward ``_csr_segment_attention_fwd`` (:62): one pass over the segment's rows in CSR order with the
  online update ``m' = max(m, l)``, ``denom = denom e^(m - m') + e^(l - m')``,
  ``acc = acc e^(m - m') + e^(l - m') v``; ``out = acc / denom`` (0 for an empty segment) and
  ``lse = m + log(denom)`` (-inf for an empty segment); a skipped segment runs no rows;
* backward ``_csr_segment_attention_bwd`` (:128): the same recurrence without ``acc`` recovers ``m`` and
  ``denom``; per row ``alpha = e^(l - m) / denom``, ``grad_value = alpha g``,
  ``grad_logits = alpha g (v - out) (+ alpha g_lse)``;
* the paired forward (:210) runs two CSRs over rows sharing ``value`` and keeps ``max`` / ``denom``;
  the paired row backward (:319) reads them per row, with the rows of a skipped segment zero.

Pinned against the reference kernels run under TRITON_INTERPRET=1 (tests/golden/segment_attention.npz,
made by tests/golden/make_golden.py): the interpreter evaluates the same FP32 operations with NumPy,
so the fixtures match this restatement to the last bit.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _rows(perm, off, s, identity, skip):
    start, end = int(off[s]), int(off[s + 1])
    if s == skip:
        end = start
    return [j if identity else int(perm[j]) for j in range(start, end)]


def _stats(logits, rows, D):
    m = np.full(D, -np.inf, F32)
    denom = np.zeros(D, F32)
    for row in rows:
        logit = logits[row]
        m_new = np.maximum(m, logit)
        denom = denom * np.exp(m - m_new) + np.exp(logit - m_new)
        m = m_new
    return m, denom


def forward(logits, value, perm, off, *, identity=False, skip=-1):
    """(out, lse, max, denom), each [S, D] float32."""
    logits, value = np.asarray(logits, F32), np.asarray(value, F32)
    S, D = len(off) - 1, logits.shape[1]
    out = np.zeros((S, D), F32)
    lse = np.full((S, D), -np.inf, F32)
    mx = np.full((S, D), -np.inf, F32)
    dn = np.zeros((S, D), F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        for s in range(S):
            m = np.full(D, -np.inf, F32)
            denom = np.zeros(D, F32)
            acc = np.zeros(D, F32)
            for row in _rows(perm, off, s, identity, skip):
                logit, val = logits[row], value[row]
                m_new = np.maximum(m, logit)
                old_scale = np.exp(m - m_new)
                new_scale = np.exp(logit - m_new)
                denom = denom * old_scale + new_scale
                acc = acc * old_scale + new_scale * val
                m = m_new
            live = denom > 0
            out[s] = np.where(live, acc / np.where(live, denom, F32(1)), F32(0))
            lse[s] = np.where(live, m + np.log(np.where(live, denom, F32(1))), -np.inf)
            mx[s], dn[s] = m, denom
    return out, lse, mx, dn


def backward(logits, value, out, gout, perm, off, *, identity=False, skip=-1, glse=None):
    """(grad_logits, grad_value) [rows, D]; rows outside every visited segment stay 0."""
    logits, value = np.asarray(logits, F32), np.asarray(value, F32)
    S, D = len(off) - 1, logits.shape[1]
    gl = np.zeros_like(logits)
    gv = np.zeros_like(value)
    with np.errstate(divide="ignore", invalid="ignore"):
        for s in range(S):
            rows = _rows(perm, off, s, identity, skip)
            m, denom = _stats(logits, rows, D)
            inv = np.where(denom > 0, F32(1) / np.where(denom > 0, denom, F32(1)), F32(0)).astype(F32)
            go, o = gout[s].astype(F32), out[s].astype(F32)
            for row in rows:
                alpha = np.exp(logits[row] - m) * inv
                gv[row] = alpha * go
                g = alpha * go * (value[row] - o)
                if glse is not None:
                    g = g + alpha * glse[s].astype(F32)
                gl[row] = g
    return gl, gv


def paired_backward_rows(la, lb, value, ga, gb, out_a, out_b, max_a, den_a, max_b, den_b, seg_a, seg_b, *,
                         skip=-1, glse_a=None, glse_b=None):
    """(grad_logits_a, grad_logits_b, grad_value) of the paired row backward."""
    la, lb, value = (np.asarray(x, F32) for x in (la, lb, value))
    gla, glb, gv = np.zeros_like(la), np.zeros_like(lb), np.zeros_like(value)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for row in range(la.shape[0]):
            sa, sb = int(seg_a[row]), int(seg_b[row])
            ia = np.where(den_a[sa] > 0, F32(1) / np.where(den_a[sa] > 0, den_a[sa], F32(1)), F32(0)).astype(F32)
            ib = np.where(den_b[sb] > 0, F32(1) / np.where(den_b[sb] > 0, den_b[sb], F32(1)), F32(0)).astype(F32)
            alpha_a = np.exp(la[row] - max_a[sa]) * ia
            alpha_b = np.exp(lb[row] - max_b[sb]) * ib
            live_a, live_b = sa != skip, sb != skip
            term_a = alpha_a * ga[sa] if live_a else np.zeros_like(alpha_a)
            term_b = alpha_b * gb[sb] if live_b else np.zeros_like(alpha_b)
            ga_row = term_a * (value[row] - out_a[sa])
            gb_row = term_b * (value[row] - out_b[sb])
            if glse_a is not None:
                ga_row = ga_row + alpha_a * glse_a[sa]
                gb_row = gb_row + alpha_b * glse_b[sb]
            gla[row] = ga_row if live_a else 0
            glb[row] = gb_row if live_b else 0
            gv[row] = term_a + term_b
    return gla, glb, gv
