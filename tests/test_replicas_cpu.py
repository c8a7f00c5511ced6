"""Replica sharding and the thermo-log gather on world_size-2 gloo groups (CPU), including a rank
that leaves before the collective (its peer's gather fails with an error, not a hang)."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, per_gpu, mode, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    from fastmd_b200.replicas import ThermoLog, replica_seeds

    try:
        seeds = replica_seeds(rank, world, per_gpu)
        log = ThermoLog(per_gpu, "cpu")
        if mode == "dead" and rank == 1:
            results[rank] = ("left", seeds)
            return  # leaves between steps, before the collective: its peer must not hang
        energies = torch.tensor([100.0 * s for s in seeds], dtype=torch.float64)
        temps = torch.tensor([500.0 + s for s in seeds], dtype=torch.float64)
        try:
            frame = log.gather(energies, temps)
            results[rank] = ("ok", frame.tolist(), seeds)
        except Exception as error:  # noqa: BLE001 - the dead-peer case reports the error
            results[rank] = ("error", type(error).__name__)
    finally:
        if not (mode == "dead" and rank == 1):
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(mode, per_gpu=3, world=2):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, per_gpu, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank hung")
    return dict(results)


def test_replica_seeds_partition():
    from fastmd_b200.replicas import replica_seeds

    seeds = [s for r in range(8) for s in replica_seeds(r, 8, 64)]
    assert sorted(seeds) == list(range(512))
    with pytest.raises(ValueError):
        replica_seeds(2, 2, 4)


def test_thermo_gather_world2():
    res = _run("ok")
    expected = [[100.0 * s, 500.0 + s] for s in range(6)]
    for rank in (0, 1):
        status, frame, seeds = res[rank]
        assert status == "ok" and frame == expected
        assert seeds == [rank * 3 + r for r in range(3)]


def test_dead_rank_fails_the_gather_without_hanging():
    res = _run("dead")
    assert res[1][0] == "left"
    assert res[0][0] == "error"
