"""Reverse-edge pairing and the line graph on the GPU against the reference's functions (golden
vectors) and the oracle on a larger random graph: integer work, bitwise."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import line_graph as olg
from oracle import neighbors as onb

pytestmark = pytest.mark.gpu


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("tag", ["perov", "triclinic", "sparse"])
def test_pairs_and_triplets_match_reference(tag):
    from fastmd_b200.line_graph import build_d2u, build_line_graph

    z = golden("line_graph")
    g = {k[len(f"plg_{tag}_"):]: z[k] for k in z if k.startswith(f"plg_{tag}_")}
    n, presorted = (int(v) for v in g["meta"])
    for sorted_flag in sorted({bool(presorted), False}):  # the sort path also on presorted input
        d2u, u2d = build_d2u(_t(g["center"]), _t(g["neighbor"]), _t(g["images"]), n, presorted=sorted_flag)
        np.testing.assert_array_equal(d2u.cpu().numpy(), g["d2u"])
        np.testing.assert_array_equal(u2d.cpu().numpy(), g["u2d"])
        tri = build_line_graph(_t(g["center"]), d2u, _t(g["dist"]), n, float(g["cutoff"][0]), presorted=sorted_flag,
                               capacity=7)  # a small first capacity: the overflow-and-grow path
        np.testing.assert_array_equal(tri.cpu().numpy(), g["triplets"])


def test_random_box_against_oracle():
    from fastmd_b200.line_graph import build_d2u, build_line_graph

    rng = np.random.default_rng(9)
    n = 300
    cell = np.eye(3) * 15.0
    pos = rng.uniform(0, 15.0, (n, 3))
    pairs = onb.dense_pairs(pos, cell, 5.0)
    keys = sorted(pairs)
    order = rng.permutation(len(keys))
    center = np.array([k[0] for k in keys], np.int64)[order]
    neighbor = np.array([k[1] for k in keys], np.int64)[order]
    images = np.array([k[2:] for k in keys], np.int32)[order]
    dist = np.array([pairs[k] for k in keys], np.float32)[order]
    d2u_ref, u2d_ref = olg.build_d2u(center, neighbor, images, n)
    d2u, u2d = build_d2u(_t(center), _t(neighbor), _t(images), n)
    np.testing.assert_array_equal(d2u.cpu().numpy(), d2u_ref)
    np.testing.assert_array_equal(u2d.cpu().numpy(), u2d_ref)
    tri = build_line_graph(_t(center), d2u, _t(dist), n, 3.0)
    np.testing.assert_array_equal(tri.cpu().numpy(), olg.build_line_graph(center, d2u_ref, dist, n, 3.0))
