"""The gated-LN epilogue on the GPU against the reference's 2-D kernels (golden vectors): the same FP32
formulas with the row sums in another order, rtol/atol 2e-6 forward and 1e-5 backward (a mean of D
products subtracted from each term)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import gated_ln as ogl

pytestmark = pytest.mark.gpu


def _t(x, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.requires_grad_(True) if grad else t


@pytest.mark.parametrize("tag", ["w128_res_bias", "w32", "w24_bias", "w128_res"])
def test_gated_ln_matches_reference_kernels(tag):
    from fastmd_b200.gated_ln import fused_gated_ln, fused_gated_ln_residual

    z = golden("gated_ln")
    g = {k[len(f"gln_{tag}_"):]: z[k] for k in z if k.startswith(f"gln_{tag}_")}
    rows, D, res, bias = (int(v) for v in g["meta"])
    cx, gx = _t(g["cx"], True), _t(g["gx"], True)
    params = [_t(g[k]) for k in ("cw", "cb", "gw", "gb")]
    kw = dict(core_lb=_t(g["clb"], True), gate_lb=_t(g["glb"], True)) if bias else {}
    if res:
        r = _t(g["res"], True)
        y = fused_gated_ln_residual(cx, gx, *params, r, _t(g["rw"]), **kw)
    else:
        y = fused_gated_ln(cx, gx, *params, **kw)
    np.testing.assert_allclose(y.detach().cpu().numpy(), g["out"], rtol=2e-6, atol=2e-6)
    inputs = [cx, gx] + ([r] if res else []) + ([kw["core_lb"], kw["gate_lb"]] if bias else [])
    grads = torch.autograd.grad(y, inputs, _t(g["g"]))
    np.testing.assert_allclose(grads[0].cpu().numpy(), g["gcore"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(grads[1].cpu().numpy(), g["ggate"], rtol=1e-5, atol=1e-5)
    if res:
        np.testing.assert_array_equal(grads[2].cpu().numpy(), g["gres"])
    if bias:  # the folded biases' gradients are the column sums of the inputs' gradients
        np.testing.assert_allclose(grads[-2].cpu().numpy(), g["gcore"].sum(0), rtol=1e-5, atol=1e-4)
        np.testing.assert_allclose(grads[-1].cpu().numpy(), g["ggate"].sum(0), rtol=1e-5, atol=1e-4)


def test_large_rows_against_oracle():
    from fastmd_b200.gated_ln import fused_gated_ln

    rng = np.random.default_rng(2)
    rows, D = 20_000, 128
    cx = rng.standard_normal((rows, D)).astype(np.float32)
    gx = rng.standard_normal((rows, D)).astype(np.float32)
    cw, cb, gw, gb = (rng.standard_normal(D).astype(np.float32) for _ in range(4))
    y = fused_gated_ln(_t(cx), _t(gx), _t(cw), _t(cb), _t(gw), _t(gb)).cpu().numpy()
    np.testing.assert_allclose(y, ogl.forward(cx, gx, cw, cb, gw, gb)[0], rtol=5e-6, atol=5e-6)


def test_errors():
    from fastmd_b200._lib import FastMDLibraryError
    from fastmd_b200.gated_ln import fused_gated_ln

    x = torch.zeros(4, 8, device="cuda")
    p = torch.ones(8, device="cuda")
    with pytest.raises(ValueError):
        fused_gated_ln(x, torch.zeros(4, 9, device="cuda"), p, p, p, p)
    with pytest.raises(FastMDLibraryError):
        fused_gated_ln(x, x, p.clone().requires_grad_(True), p, p, p)
