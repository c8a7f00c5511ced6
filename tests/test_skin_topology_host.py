"""Host logic of the skin-epoch topology runner (no device)."""
import numpy as np
import pytest

from fastmd_b200.skin_topology import PROACTIVE_REFRESH_FRACTION, SkinTopologyRunner


def test_minimum_image_displacement():
    runner = object.__new__(SkinTopologyRunner)
    runner.cell = np.diag([10.0, 12.0, 14.0])
    runner._inv_cell = np.linalg.inv(runner.cell)
    runner._reference = np.zeros((3, 3))
    moved = np.array([[9.9, 0.0, 0.0], [0.0, 0.3, 0.0], [0.0, 0.0, 14.0]])  # a wrap is no motion
    assert runner._displacement(moved) == pytest.approx(0.3)
    assert 0 < PROACTIVE_REFRESH_FRACTION < 0.5


def test_skin_must_be_positive():
    with pytest.raises(ValueError):
        SkinTopologyRunner(None, atomic_numbers=[1], cell=np.eye(3), skin=0.0)
