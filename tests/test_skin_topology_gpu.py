"""The skin-epoch topology runner (fastmd/execution/skin_topology.py:93) on the GPU: every evaluation equals
the model's evaluation of a fresh fixed-capacity build of the same positions, bit for bit, across refreshes,
captured or eager, and after the redo paths (a skin violation the host did not see, a bucket too small)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _system(seed=0):
    from fastmd_b200.structures import perovskite

    pos, cell, numbers, _ = perovskite(seed=seed)
    return pos, cell, numbers


def _fresh(model, pos, cell, numbers, cuda):
    """Energy and forces of a fresh build (own candidates) of ``pos``."""
    from fastmd_b200.graph import FixedCapacityGraphBuilder

    b = FixedCapacityGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32), atomic_numbers=torch.tensor(numbers),
                                  u_capacity=1400, atom_graph_cutoff=6.0, candidate_cutoff=7.0, device=cuda,
                                  minimum_image=True)
    batch, status = b.build(torch.from_numpy(np.asarray(pos, np.float32)).to(cuda))
    assert int(status.flags.item()) == 0
    e, f = model.energy_forces_fused(model.prepare(batch))
    return float(e[0]), f.cpu().numpy()


def _runner(model, cell, numbers, cuda, **kw):
    from fastmd_b200.skin_topology import SkinTopologyRunner

    return SkinTopologyRunner(model, atomic_numbers=numbers, cell=cell, skin=kw.pop("skin", 1.0), device=cuda, **kw)


@pytest.mark.parametrize("capture", [True, False])
def test_evaluations_equal_fresh_builds(cuda, capture):
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers = _system()
    model = MACEModel(device=cuda)
    runner = _runner(model, cell, numbers, cuda, capture=capture, u_step=64, min_pad_u=16)
    rng = np.random.default_rng(4)
    p = pos.copy()
    for _ in range(10):
        p = p + rng.normal(0.0, 0.08, p.shape)
        got = runner.evaluate(p)
        e, f = _fresh(model, p, cell, numbers, cuda)
        assert got["e"] == e and np.array_equal(got["f"], f)
    st = runner.stats()
    assert st["calls"] == 10 and st["refreshes"] >= 2 and st["redo_skin"] == 0
    assert (st["captures"] >= 1) == capture
    runner.close()


def test_a_skin_violation_is_redone(cuda, monkeypatch):
    from fastmd_b200 import skin_topology
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers = _system(1)
    model = MACEModel(device=cuda)
    runner = _runner(model, cell, numbers, cuda)
    runner.evaluate(pos)
    monkeypatch.setattr(skin_topology, "PROACTIVE_REFRESH_FRACTION", 100.0)  # the host never refreshes
    moved = pos.copy()
    moved[7] += (0.7, 0.0, 0.0)  # more than half the skin (0.5 A)
    got = runner.evaluate(moved)
    assert runner.redo_skin == 1 and runner.refreshes == 2
    e, f = _fresh(model, moved, cell, numbers, cuda)
    assert got["e"] == e and np.array_equal(got["f"], f)
    runner.close()


def test_a_bucket_too_small_is_redone(cuda):
    from fastmd_b200.mace import MACEModel

    pos, cell, numbers = _system(2)
    model = MACEModel(device=cuda)
    runner = _runner(model, cell, numbers, cuda, u_step=1, min_pad_u=0)
    runner.evaluate(pos)
    runner.close()
    runner._demand = 10  # a stale demand: its bucket holds 11 pairs
    p = pos + 0.01
    got = runner.evaluate(p)
    assert runner.redo_capacity == 1
    assert runner.last_edge_count == 2 * runner._demand
    e, f = _fresh(model, p, cell, numbers, cuda)
    assert got["e"] == e and np.array_equal(got["f"], f)
    runner.close()


def test_truncated_candidate_rows_raise(cuda):
    from fastmd_b200.mace import MACEModel
    from fastmd_b200.skin_topology import SkinTopologyUnavailable

    pos, cell, numbers = _system()
    runner = _runner(MACEModel(device=cuda), cell, numbers, cuda, max_neighbors=16)
    with pytest.raises(SkinTopologyUnavailable):
        runner.evaluate(pos)
