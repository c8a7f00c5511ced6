"""The residual-add oracle against the reference kernels' golden outputs (bitwise)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import residual_add as ora

GOLDEN = np.load(Path(__file__).parent / "golden" / "residual_add.npz")
TAGS = ["d128", "d64_strided", "d5"]


@pytest.mark.parametrize("tag", TAGS)
def test_forward_and_backward_bitwise(tag):
    n, d, _, _ = (int(v) for v in GOLDEN[f"ra_{tag}_meta"])
    delta = GOLDEN[f"ra_{tag}_delta"][:, :d]
    residual = GOLDEN[f"ra_{tag}_residual"][:, :d]
    weight = GOLDEN[f"ra_{tag}_weight"]
    np.testing.assert_array_equal(ora.forward(delta, residual, weight), GOLDEN[f"ra_{tag}_out"])
    gd, gr = ora.backward(GOLDEN[f"ra_{tag}_gout"], weight)
    np.testing.assert_array_equal(gd, GOLDEN[f"ra_{tag}_gout"])
    np.testing.assert_array_equal(gr, GOLDEN[f"ra_{tag}_gres"])
    assert gr.shape == (n, d)


def test_oracle_catches_a_fused_product():
    """A fused multiply-add (one rounding) differs from the reference's two roundings on some inputs:
    the pin is not vacuous."""
    rng = np.random.default_rng(0)
    d, r, w = (rng.standard_normal(4096).astype(np.float32) for _ in range(3))
    fused = (d.astype(np.float64) + r.astype(np.float64) * w.astype(np.float64)).astype(np.float32)
    assert np.any(fused != ora.forward(d[None], r[None], w)[0])
