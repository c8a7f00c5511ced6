"""Segment attention on the GPU against the reference's kernels (golden vectors of the Triton kernels
run by the interpreter) and the oracle. Tolerance: the recurrence is the reference's FP32 program
operation for operation (no contraction); expf/logf differ from NumPy's by an ulp or two, which the
online rescaling carries along: rtol 2e-6 + atol 2e-6 (5e-6 on gradients)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import segment_attention as osa

pytestmark = pytest.mark.gpu
RTOL, ATOL = 2e-6, 2e-6


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _close(a, b, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(a.detach().cpu().numpy(), b, rtol=rtol, atol=atol)


@pytest.mark.parametrize("tag", ["perm_lse", "identity_skip", "odd_lse_skip", "wide_empty"])
def test_segment_attention_matches_reference_kernels(tag):
    from fastmd_b200.segment_attention import segment_attention

    z = golden("segment_attention")
    g = {k[len(f"sa_{tag}_"):]: z[k] for k in z if k.startswith(f"sa_{tag}_")}
    S, identity, skip, lse = (int(v) for v in g["meta"])
    L = _t(g["L"]).requires_grad_(True)
    V = _t(g["V"]).requires_grad_(True)
    res = segment_attention(L, V, _t(g["seg"]), S, None if identity else _t(g["perm"]), _t(g["off"]),
                            bool(identity), skip_segment=skip, return_lse=bool(lse))
    out = res[0] if lse else res
    _close(out, g["out"])
    grads = [_t(g["G"])]
    outs = [out]
    if lse:
        lse_ref = g["lse"]
        got = res[1].detach().cpu().numpy()
        assert np.array_equal(np.isneginf(got), np.isneginf(lse_ref))
        fin = np.isfinite(lse_ref)
        np.testing.assert_allclose(got[fin], lse_ref[fin], rtol=RTOL, atol=ATOL)
        outs.append(res[1])
        grads.append(_t(g["GL"]))
    gl, gv = torch.autograd.grad(outs, [L, V], grads)
    _close(gl, g["glogits"], atol=5e-6)
    _close(gv, g["gvalue"], atol=5e-6)


@pytest.mark.parametrize("tag", ["pair", "pair_skip"])
def test_paired_segment_attention_matches_reference_kernels(tag):
    from fastmd_b200.segment_attention import paired_segment_attention

    z = golden("segment_attention")
    g = {k[len(f"psa_{tag}_"):]: z[k] for k in z if k.startswith(f"psa_{tag}_")}
    S, skip, lse = (int(v) for v in g["meta"])
    La, Lb, V = (_t(g[k]).requires_grad_(True) for k in ("La", "Lb", "V"))
    res = paired_segment_attention(La, Lb, V, _t(g["sa"]), _t(g["sb"]), S, _t(g["pa"]), _t(g["oa"]), _t(g["pb"]),
                                   _t(g["ob"]), skip_segment=skip, return_lse=bool(lse))
    _close(res[0], g["out_a"])
    _close(res[1], g["out_b"])
    grads = [_t(g["Ga"]), _t(g["Gb"])]
    if lse:
        for got, ref in ((res[2], g["lse_a"]), (res[3], g["lse_b"])):
            fin = np.isfinite(ref)
            np.testing.assert_allclose(got.detach().cpu().numpy()[fin], ref[fin], rtol=RTOL, atol=ATOL)
        grads += [_t(g["GLa"]), _t(g["GLb"])]
    gla, glb, gv = torch.autograd.grad(list(res), [La, Lb, V], grads)
    _close(gla, g["glogits_a"], atol=5e-6)
    _close(glb, g["glogits_b"], atol=5e-6)
    _close(gv, g["gvalue"], atol=5e-6)


def test_larger_case_against_oracle_and_computed_csr():
    """20k rows x 128, 1,500 segments (some empty), the CSR built on the device; then the CPU oracle."""
    from fastmd_b200.segment_attention import segment_attention

    rng = np.random.default_rng(4)
    rows, S, D = 20_000, 1500, 128
    seg = rng.integers(0, S - 100, rows).astype(np.int64)  # the last 100 segments empty
    L = (3 * rng.standard_normal((rows, D))).astype(np.float32)
    V = rng.standard_normal((rows, D)).astype(np.float32)
    out = segment_attention(_t(L), _t(V), _t(seg), S).cpu().numpy()
    perm = np.argsort(seg, kind="stable")
    off = np.searchsorted(seg[perm], np.arange(S + 1))
    ref = osa.forward(L, V, perm, off)[0]
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)
    assert not out[S - 100:].any()


def test_errors_mirror_the_reference():
    from fastmd_b200.segment_attention import segment_attention

    x = torch.zeros(4, 8, device="cuda")
    seg = torch.zeros(4, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        segment_attention(x, torch.zeros(4, 9, device="cuda"), seg, 2)
    with pytest.raises(ValueError):
        segment_attention(x, x, seg, 2, skip_segment=2)
    with pytest.raises(ValueError):
        segment_attention(x, x, seg, 2, identity_perm=True)
