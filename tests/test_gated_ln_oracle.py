"""The gated-LN oracle against the reference's 2-D kernels (golden vectors), to FP32 rounding."""
import numpy as np
import pytest

from conftest import golden
from oracle import gated_ln as ogl

CASES = ["w128_res_bias", "w32", "w24_bias", "w128_res"]


@pytest.mark.parametrize("tag", CASES)
def test_gated_ln_matches_reference(tag):
    z = golden("gated_ln")
    g = {k[len(f"gln_{tag}_"):]: z[k] for k in z if k.startswith(f"gln_{tag}_")}
    rows, D, res, bias = (int(v) for v in g["meta"])
    kw = dict(core_lb=g["clb"], gate_lb=g["glb"]) if bias else {}
    out, cmu, crs, gmu, grs = ogl.forward(g["cx"], g["gx"], g["cw"], g["cb"], g["gw"], g["gb"], **kw,
                                          residual=g["res"] if res else None, res_weight=g["rw"] if res else None)
    np.testing.assert_allclose(out, g["out"], rtol=2e-6, atol=2e-6)
    for mine, k in ((cmu, "cmean"), (crs, "crstd"), (gmu, "gmean"), (grs, "grstd")):
        np.testing.assert_allclose(mine, g[k], rtol=2e-6, atol=2e-6)
    gc, gg, gr = ogl.backward(g["cx"], g["gx"], g["cw"], g["cb"], g["gw"], g["gb"], g["g"], g["cmean"], g["crstd"],
                              g["gmean"], g["grstd"], **kw, res_weight=g["rw"] if res else None)
    np.testing.assert_allclose(gc, g["gcore"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gg, g["ggate"], rtol=1e-5, atol=1e-5)
    if res:
        np.testing.assert_array_equal(gr, g["gres"])
