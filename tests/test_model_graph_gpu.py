"""The model_graph runner on the GPU: replays of each bucket's captured fused evaluation return the eager
evaluation of the ragged build bit for bit, across builds of changing edge counts; bucket captures,
reuses and rebinds as fastmd/execution/cuda_graph.py:677 selects them."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _builds(cuda, n_builds=6, seed=0):
    from fastmd_b200.graph import TensorGraphBuilder
    from fastmd_b200.structures import perovskite

    pos, cell, numbers, _ = perovskite(seed=seed)
    builder = TensorGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32), atomic_numbers=torch.tensor(numbers),
                                 atom_graph_cutoff=6.0, device=cuda)
    rng = np.random.default_rng(seed + 11)
    out = []
    for k in range(n_builds):  # growing jitter: the edge count wanders
        p = pos + rng.normal(0.0, 0.05 + 0.08 * k, pos.shape)
        out.append(builder.build(torch.from_numpy(p.astype(np.float32)).to(cuda)))
    return out


def test_replays_match_eager_bitwise(cuda):
    from fastmd_b200.mace import MACEModel
    from fastmd_b200.model_graph import BucketedGraphRunner

    builds = _builds(cuda)
    model = MACEModel(device=cuda)
    runner = BucketedGraphRunner(model, u_step=64, min_pad_u=16)
    edges = [int(b.edge_index.shape[0]) for b in builds]
    assert len(set(edges)) > 1
    for b in builds:
        energy, forces = (x.clone() for x in runner.run(b))
        ref_e, ref_f = model.energy_forces_fused(model.prepare(b))
        assert torch.equal(energy, ref_e) and torch.equal(forces, ref_f)
    st = runner.stats()
    assert 1 <= st["captures"] <= len(builds) and st["pool_resets"] == 0
    assert all(key % 64 == 0 for key in st["cached_buckets"])
    # every build fits a cached bucket now: replays only
    captures = st["captures"]
    for b in builds:
        runner.run(b)
    assert runner.stats()["captures"] == captures


def test_rebind_on_another_system(cuda):
    from fastmd_b200.graph import TensorGraphBuilder
    from fastmd_b200.mace import MACEModel
    from fastmd_b200.model_graph import BucketedGraphRunner
    from fastmd_b200.structures import perovskite

    model = MACEModel(device=cuda)
    runner = BucketedGraphRunner(model)
    runner.run(_builds(cuda, 1)[0])
    pos, cell, numbers, _ = perovskite(seed=3)
    keep = np.arange(numbers.size) != 7  # one atom fewer
    builder = TensorGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32),
                                 atomic_numbers=torch.tensor(numbers[keep]), atom_graph_cutoff=6.0, device=cuda)
    b = builder.build(torch.from_numpy(pos[keep].astype(np.float32)).to(cuda))
    energy, forces = (x.clone() for x in runner.run(b))
    assert runner.stats()["pool_resets"] == 1 and runner.stats()["captures"] == 2
    ref_e, ref_f = model.energy_forces_fused(model.prepare(b))
    assert torch.equal(energy, ref_e) and torch.equal(forces, ref_f)
