"""The fixed-capacity bond-graph oracle against the reference builder's own outputs (bitwise)."""
import numpy as np
import pytest

from conftest import golden
from oracle import bond_graph as obg
from oracle import neighbors as onb

TAGS = ["perov_sink", "perov_loop", "perov_sink_tover", "perov_loop_eover", "tric_sink"]


def oracle_case(g, tag):
    """The oracle bond graph of a golden case, from its positions (candidates, re-filter, short flags)."""
    N, n_dummy, u_cap, t_cap, total, t_real, sink = (int(v) for v in g[f"bg_{tag}_meta"])
    rc, lrc, cand = g[f"bg_{tag}_cutoffs"]
    cell, pos = g[f"bg_{tag}_cell"], g[f"bg_{tag}_positions"]
    wrapped, _, _ = onb.wrap(pos, cell, inv_cell=onb.inverse_cell(cell))
    nm, ns, nn = onb.candidates(wrapped, cell, cand)
    c, n, im, _, short = onb.refilter(wrapped, cell, nm, ns, nn, rc, line_cutoff=lrc)
    assert c.size == total
    return obg.build(c, n, im, short, total, n_real=N, u_capacity=u_cap, t_capacity=t_cap, sink=bool(sink),
                     n_dummy=n_dummy, pad_image=g[f"bg_{tag}_pad_image"]), t_real


@pytest.mark.parametrize("tag", TAGS)
def test_oracle_equals_reference_builder(tag):
    g = golden("bond_graph")
    out, t_real = oracle_case(g, tag)
    assert out["n_triplets"] == t_real
    for key in ("center", "neighbor", "images", "d2u", "u2d", "line_graph"):
        np.testing.assert_array_equal(out[key], g[f"bg_{tag}_{key}"], err_msg=key)
    assert [out["overflow"], out["invalid_pairs"]] == g[f"bg_{tag}_flags"].tolist()


def test_a_missing_reverse_edge_is_an_invalid_pair():
    """Drop one directed edge: the pairing is invalid, the build overflows onto the padding topology."""
    g = golden("bond_graph")
    N, n_dummy, u_cap, t_cap, total, _, _ = (int(v) for v in g["bg_perov_sink_meta"])
    cell, pos = g["bg_perov_sink_cell"], g["bg_perov_sink_positions"]
    wrapped, _, _ = onb.wrap(pos, cell, inv_cell=onb.inverse_cell(cell))
    c, n, im, _, short = onb.refilter(wrapped, cell, *onb.candidates(wrapped, cell, 8.0), 6.0, line_cutoff=4.5)
    keep = np.arange(c.size) != 17
    out = obg.build(c[keep], n[keep], im[keep], short[keep], total - 1, n_real=N, u_capacity=u_cap,
                    t_capacity=t_cap, sink=True, n_dummy=n_dummy)
    assert out["invalid_pairs"] and out["overflow"]
    assert np.array_equal(out["d2u"], np.arange(2 * u_cap) // 2)
