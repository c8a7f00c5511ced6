"""The float64 build-prologue oracle against the reference kernel's golden outputs (bitwise)."""
import numpy as np
import pytest

from conftest import golden
from oracle import neighbors as onb


@pytest.mark.parametrize("tag", ["tric", "cubic"])
def test_float64_prologue_bitwise(tag):
    g = golden("float64")
    out = onb.float64_prologue(g[f"f64_{tag}_positions"], g[f"f64_{tag}_cell"],
                               g[f"f64_{tag}_reference"].astype(np.float32), g[f"f64_{tag}_ref_wraps"],
                               float(g[f"f64_{tag}_skin"][0]), inv_cell=g[f"f64_{tag}_inv32"])
    for key in ("wrapped", "frac", "model_positions", "wrap_delta"):
        np.testing.assert_array_equal(out[key], g[f"f64_{tag}_{key}"], err_msg=key)
    assert out["max_displacement"] == g[f"f64_{tag}_max_displacement"][0]
    assert out["candidate_valid"] == bool(g[f"f64_{tag}_candidate_valid"][0])
    # the float32 inverse is the float64 inverse rounded once
    np.testing.assert_array_equal(onb.inverse_cell(g[f"f64_{tag}_cell"].astype(np.float32)), g[f"f64_{tag}_inv32"])
