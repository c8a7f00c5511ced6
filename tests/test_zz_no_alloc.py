"""The allocation-free re-filter entry point against the workspace one.

``fmd_refilter_edges_noalloc`` serves callers that cannot allocate device
memory (a C or Fortran MD host without a CUDA allocator of its own, or a
caller inside another framework's memory manager): its scratch is a static
device array inside the library. Here it is called through the C ABI on the
same candidates and positions as ``fmd_refilter_edges`` (through the
builder), twice in a row with different positions, and every output must be
bit-identical. This file is collected last so that a run stopping at the
first failure has run every other test; it also passes alone.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_build(builder, positions):
    """The builder's per-step build, through the allocation-free entry point, into fresh buffers."""
    from fastmd_b200._lib import call, ptr, stream

    dev = builder.device
    N, E = builder.n_real, builder.e_capacity
    out = {
        "wrapped": torch.full((N, 3), float("nan"), device=dev),
        "wrap_delta": torch.full((N, 3), -7, dtype=torch.int32, device=dev),
        "edge_index": torch.full((E, 2), -7, dtype=torch.int32, device=dev),
        "edge_image": torch.full((E, 3), float("nan"), device=dev),
        "recv_off": torch.full((N + 1,), -7, dtype=torch.int64, device=dev),
        "send_off": torch.full((N + 1,), -7, dtype=torch.int64, device=dev),
        "send_perm": torch.full((E,), -7, dtype=torch.int32, device=dev),
        "n_edges": torch.full((1,), -7, dtype=torch.int64, device=dev),
        "max_displacement": torch.full((builder.replicas,), float("nan"), device=dev),
        "flags": builder.refresh_flags.clone(),
    }
    pos = positions.contiguous()
    call("fmd_refilter_edges_noalloc", ptr(pos), builder._cell_ptr, builder.n_atoms, builder.replicas,
         ptr(builder.reference_positions), ptr(builder.reference_wraps), ptr(builder.cand_nbr),
         ptr(builder.cand_shift), ptr(builder.cand_count), builder.buffer_max, builder.atom_graph_cutoff,
         builder.skin, E, builder._pad_image_host, int(builder.minimum_image), ptr(out["wrapped"]),
         ptr(out["wrap_delta"]), ptr(out["edge_index"]), ptr(out["edge_image"]), ptr(out["recv_off"]),
         ptr(out["send_off"]), ptr(out["send_perm"]), ptr(out["n_edges"]), ptr(out["max_displacement"]),
         ptr(out["flags"]), stream(dev))
    torch.cuda.synchronize()
    return out


def _compare(builder, out):
    b = builder.batch
    n = int(b.n_edges.item())
    assert int(out["n_edges"].item()) == n
    assert torch.equal(out["wrapped"], b.positions)
    assert torch.equal(out["wrap_delta"], builder.wrap_delta)
    assert torch.equal(out["edge_index"], b.edge_index)
    assert torch.equal(out["edge_image"], b.edge_image)
    assert torch.equal(out["recv_off"], b.recv_off)
    assert torch.equal(out["send_off"], b.send_off)
    assert torch.equal(out["send_perm"][:n], b.send_perm[:n])
    assert torch.equal(out["max_displacement"], builder.max_displacement)
    assert torch.equal(out["flags"], builder.flags)


@pytest.mark.parametrize("replicas", [1, 3])
def test_noalloc_refilter_equals_workspace_refilter_twice(cuda, replicas):
    from fastmd_b200.graph import FixedCapacityGraphBuilder
    from fastmd_b200.structures import perovskite

    systems = [perovskite(seed=s) for s in range(replicas)]
    cell, numbers = systems[0][1], systems[0][2]
    pos = torch.from_numpy(np.concatenate([s[0] for s in systems]).astype(np.float32)).to(cuda)
    builder = FixedCapacityGraphBuilder(cell=torch.tensor(cell, dtype=torch.float32),
                                        atomic_numbers=torch.tensor(numbers), u_capacity=1200 * replicas,
                                        atom_graph_cutoff=6.0, candidate_cutoff=8.0, device=cuda,
                                        replicas=replicas)
    builder.refresh_candidates(pos)
    gen = torch.Generator(device=cuda).manual_seed(11)
    for call_index in range(2):  # two calls in a row share (and overwrite) the static scratch
        moved = pos + 0.3 * (torch.rand(pos.shape, device=cuda, generator=gen) - 0.5)
        builder.build(moved, rebuild_candidates=False)
        torch.cuda.synchronize()
        assert int(builder.flags.item()) == 0
        _compare(builder, _noalloc_build(builder, moved))


def test_noalloc_refilter_rejects_sizes_beyond_the_scratch(cuda):
    from fastmd_b200._lib import lib

    cell = (ctypes.c_float * 9)(20, 0, 0, 0, 20, 0, 0, 0, 20)
    one = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    status = lib().fmd_refilter_edges_noalloc(
        one, ctypes.cast(cell, ctypes.c_void_p), 126_977, 1, one, one, one, one, one, 16, 6.0, 2.0, 1024, None,
        0, one, one, one, one, one, one, one, one, one, one, None)
    assert status == 4  # FMD_ERR_WORKSPACE
    status = lib().fmd_refilter_edges_noalloc(
        one, ctypes.cast(cell, ctypes.c_void_p), 2_000, 100, one, one, one, one, one, 16, 6.0, 2.0, 1024, None,
        0, one, one, one, one, one, one, one, one, one, one, None)
    assert status == 4


def test_refilter_on_a_second_device_after_the_first():
    """The dynamic shared-memory limit a launch raises applies to the current device only: a re-filter of a
    system above 2,048 atoms (beyond the default 48 KB) on device 1 after one on device 0 must raise it again
    there, for the workspace entry point and the allocation-free one, and give the same bits on both."""
    from fastmd_b200.graph import FixedCapacityGraphBuilder

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    n, box = 3000, (3000 / 0.06) ** (1.0 / 3.0)
    pos = torch.from_numpy(np.random.default_rng(4).uniform(0.0, box, (n, 3)).astype(np.float32))
    cell = torch.eye(3) * box
    results = []
    for index in (0, 1):
        dev = torch.device(f"cuda:{index}")
        with torch.cuda.device(dev):
            builder = FixedCapacityGraphBuilder(cell=cell, atomic_numbers=torch.full((n,), 14), u_capacity=120_000,
                                                atom_graph_cutoff=6.0, candidate_cutoff=6.5, device=dev)
            p = pos.to(dev)
            builder.refresh_candidates(p)
            builder.build(p, rebuild_candidates=False)
            torch.cuda.synchronize(dev)
            assert int(builder.flags.item()) == 0
            _compare(builder, _noalloc_build(builder, p))
            m = int(builder.batch.n_edges.item())
            results.append((builder.batch.edge_index[:m].cpu(), builder.batch.edge_image[:m].cpu()))
    assert torch.equal(results[0][0], results[1][0]) and torch.equal(results[0][1], results[1][1])
