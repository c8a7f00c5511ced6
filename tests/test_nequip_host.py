"""Host logic of the NequIP-architecture model (no kernel launches)."""
import numpy as np
import pytest

from fastmd_b200 import nequip
from fastmd_b200._lib import FastMDLibraryError
from oracle import nequip as onq


def test_layout_constants():
    assert len(nequip.PATHS) == 15 and nequip.PATHS == onq.PATHS
    assert (nequip.X_WIDTH, nequip.M_MULT, nequip.W_WIDTH) == (480, (224, 384, 352), 960)


def test_coupling_table_is_the_oracles_and_deterministic():
    table = nequip.coupling_table()
    assert table.shape == (615,) and table.dtype == np.float32
    ref = np.concatenate([onq.clebsch_gordan(*p).reshape(-1) for p in onq.PATHS]).astype(np.float32)
    np.testing.assert_array_equal(table, ref)
    np.testing.assert_array_equal(table, nequip.coupling_table())


def test_weights_shapes():
    cfg = nequip.NequIPConfig(num_layers=2)
    w = nequip.init_weights(cfg, seed=4)
    assert w["embed"].shape == (89, 128) and w["L1.rad3"].shape == (960, 64)
    assert w["L0.sc1"].shape == (89, 64, 64) and w["L0.lin2_0"].shape == (224, 224)
    assert w["L1.lin2_2"].shape == (352, 32) and w["readout2"].shape == (1, 64)
    assert all(v.dtype == np.float32 for v in w.values())


def test_no_cpu_model():
    with pytest.raises(FastMDLibraryError):
        nequip.NequIPModel(nequip.NequIPConfig(num_layers=1), device="cpu")
