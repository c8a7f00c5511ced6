"""The gather-add-SiLU oracle against the reference's epilogue kernels (golden vectors)."""
import numpy as np
import pytest

from conftest import golden
from oracle import gather_add_silu as ogas


@pytest.mark.parametrize("tag", ["cat3", "cat3_sorted_odd", "cat4"])
def test_gather_add_silu_matches_reference(tag):
    z = golden("gather_add_silu")
    g = {k[len(f"gas_{tag}_"):]: z[k] for k in z if k.startswith(f"gas_{tag}_")}
    M, NS, H, cat4, _, bias = (int(v) for v in g["meta"])
    parts = [(g["p1"], g["ia"]), (g["p2"], g["ib"])] + ([(g["p3"], g["ic"])] if cat4 else [])
    pre, core, gate = ogas.forward(g["p0"], parts, g["b"] if bias else None)
    np.testing.assert_array_equal(pre, g["preact"])
    np.testing.assert_array_equal(core, g["core"])
    np.testing.assert_array_equal(gate, g["gate"])
    gp0, gps = ogas.backward(g["gc"], g["gg"], g["preact"], [(NS, idx) for _, idx in parts])
    np.testing.assert_array_equal(gp0, g["gp0"])
    for k, gk in enumerate(gps, start=1):
        np.testing.assert_allclose(gk, g[f"gp{k}"], rtol=1e-6, atol=1e-6)
