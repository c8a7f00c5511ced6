"""The pair-aggregation oracle against the reference's kernels (golden vectors), bitwise."""
import numpy as np
import pytest

from conftest import golden
from oracle import pair_aggregate as opa

CASES = ["d32", "d128_strided", "d5"]


@pytest.mark.parametrize("tag", CASES)
def test_pair_aggregate_matches_reference(tag):
    z = golden("pair_aggregate")
    g = {k[len(f"pa_{tag}_"):]: z[k] for k in z if k.startswith(f"pa_{tag}_")}
    U, D, stride = (int(v) for v in g["meta"])
    assert g["base"].shape == (2 * U, stride) and g["pair"].shape == (U, 2)
    np.testing.assert_array_equal(opa.average(g["base"][:, :D], g["pair"]), g["avg"])
    np.testing.assert_array_equal(opa.average_bwd(g["gavg"], g["pair"], 2 * U), g["gdata"])
    np.testing.assert_array_equal(opa.expand(g["und"][:, :D], g["pair"], 2 * U), g["exp"])
    np.testing.assert_array_equal(opa.expand_bwd(g["gexp"], g["pair"]), g["gund"])


def test_pair_index_is_a_bijection():
    z = golden("pair_aggregate")
    for tag in CASES:
        pair = z[f"pa_{tag}_pair"]
        assert np.array_equal(np.sort(pair.ravel()), np.arange(pair.size))
