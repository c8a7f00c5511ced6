"""The reverse-pairing / line-graph oracle against the reference's own functions (golden vectors)."""
import numpy as np
import pytest

from conftest import golden
from oracle import line_graph as olg


@pytest.mark.parametrize("tag", ["perov", "triclinic", "sparse"])
def test_pairs_and_triplets_match_reference(tag):
    z = golden("line_graph")
    g = {k[len(f"plg_{tag}_"):]: z[k] for k in z if k.startswith(f"plg_{tag}_")}
    n, presorted = (int(v) for v in g["meta"])
    d2u, u2d = olg.build_d2u(g["center"], g["neighbor"], g["images"], n, presorted=bool(presorted))
    np.testing.assert_array_equal(d2u, g["d2u"])
    np.testing.assert_array_equal(u2d, g["u2d"])
    tri = olg.build_line_graph(g["center"], g["d2u"], g["dist"], n, float(g["cutoff"][0]), presorted=bool(presorted))
    np.testing.assert_array_equal(tri, g["triplets"])
    # every directed edge is paired with its reverse: two edges per undirected edge
    assert np.all(np.bincount(d2u) == 2)
