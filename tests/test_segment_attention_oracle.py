"""The segment-attention oracle against the reference's own kernels (run under the Triton
interpreter into tests/golden/segment_attention.npz): bitwise."""
import numpy as np
import pytest

from oracle import segment_attention as osa
from conftest import golden as _golden

CASES = ["perm_lse", "identity_skip", "odd_lse_skip", "wide_empty"]


@pytest.mark.parametrize("tag", CASES)
def test_segment_attention_matches_reference(tag):
    z = _golden("segment_attention")
    g = {k[len(f"sa_{tag}_"):]: z[k] for k in z if k.startswith(f"sa_{tag}_")}
    S, identity, skip, lse = (int(v) for v in g["meta"])
    out, ls, _, _ = osa.forward(g["L"], g["V"], g["perm"], g["off"], identity=bool(identity), skip=skip)
    np.testing.assert_array_equal(out, g["out"])
    if lse:
        np.testing.assert_array_equal(ls, g["lse"])
    gl, gv = osa.backward(g["L"], g["V"], g["out"], g["G"], g["perm"], g["off"], identity=bool(identity), skip=skip,
                          glse=g["GL"] if lse else None)
    np.testing.assert_array_equal(gl, g["glogits"])
    np.testing.assert_array_equal(gv, g["gvalue"])
    if skip >= 0:  # the skipped segment: out 0, its rows get no gradient
        assert not out[skip].any()
        rows = g["perm"][g["off"][skip]:g["off"][skip + 1]] if not identity else np.arange(g["off"][skip], g["off"][skip + 1])
        assert not gl[rows].any() and not gv[rows].any()


@pytest.mark.parametrize("tag", ["pair", "pair_skip"])
def test_paired_segment_attention_matches_reference(tag):
    z = _golden("segment_attention")
    g = {k[len(f"psa_{tag}_"):]: z[k] for k in z if k.startswith(f"psa_{tag}_")}
    S, skip, lse = (int(v) for v in g["meta"])
    for side in ("a", "b"):
        out, ls, mx, dn = osa.forward(g[f"L{side}"], g["V"], g[f"p{side}"], g[f"o{side}"], skip=skip)
        np.testing.assert_array_equal(out, g[f"out_{side}"])
        np.testing.assert_array_equal(mx, g[f"max_{side}"])
        np.testing.assert_array_equal(dn, g[f"denom_{side}"])
        if lse:
            np.testing.assert_array_equal(ls, g[f"lse_{side}"])
    gla, glb, gv = osa.paired_backward_rows(
        g["La"], g["Lb"], g["V"], g["Ga"], g["Gb"], g["out_a"], g["out_b"], g["max_a"], g["denom_a"], g["max_b"],
        g["denom_b"], g["sa"], g["sb"], skip=skip, glse_a=g["GLa"] if lse else None, glse_b=g["GLb"] if lse else None)
    np.testing.assert_array_equal(gla, g["glogits_a"])
    np.testing.assert_array_equal(glb, g["glogits_b"])
    np.testing.assert_array_equal(gv, g["gvalue"])
