"""The padding-row oracle against the reference's ``_pad_self_loops_kernel`` golden rows (bitwise), and
the exact-rc padding rule's host checks."""
import numpy as np
import pytest

from conftest import golden
from oracle import neighbors as onb


@pytest.mark.parametrize("tag", ["far", "exact_rc"])
def test_padding_rows_bitwise(tag):
    g = golden("padding")
    total, e_cap, n = (int(v) for v in g[f"pad_{tag}_meta"])
    c, nb, im = onb.pad_self_loops(total, e_cap, n, g[f"pad_{tag}_image"])
    np.testing.assert_array_equal(c, g[f"pad_{tag}_center"][total:])
    np.testing.assert_array_equal(nb, g[f"pad_{tag}_neighbor"][total:])
    np.testing.assert_array_equal(im, g[f"pad_{tag}_images"][total:])
    if tag == "exact_rc":
        np.testing.assert_array_equal(onb.pad_vector_override(total, e_cap, g[f"pad_{tag}_vector"]),
                                      g[f"pad_{tag}_override"])


def test_exact_rc_rule_checks():
    from fastmd_b200.graph import PaddingRule, exact_rc_pad_vector

    assert exact_rc_pad_vector(PaddingRule("exact_rc_loops"), 5.0) == (5.0, 0.0, 0.0)
    assert exact_rc_pad_vector(PaddingRule("exact_rc_loops", pad_vector=(3.0, 4.0, 0.0)), 5.0) == (3.0, 4.0, 0.0)
    with pytest.raises(ValueError):
        exact_rc_pad_vector(PaddingRule("exact_rc_loops", pad_vector=(4.9, 0.0, 0.0)), 5.0)
    with pytest.raises(ValueError):
        PaddingRule("far_self_loops", pad_vector=(5.0, 0.0, 0.0))
    with pytest.raises(ValueError):
        PaddingRule("exact_rc_loops", min_length=3.0)
