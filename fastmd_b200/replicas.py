"""Replica sharding across GPUs (replica_md.py:224 runs them on one GPU).

Independent trajectory replicas shard with no exchange on the step path: rank r of W integrates
``per_gpu`` replicas with seeds ``r*per_gpu .. r*per_gpu + per_gpu - 1`` as one disjoint-union
graph on its own GPU. The only collective is the thermo log: every ``log_every`` steps the
per-replica (E_pot, T) of all ranks are all-gathered (NCCL over NVLink on GPUs, gloo on CPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def replica_seeds(rank: int, world: int, per_gpu: int) -> list[int]:
    """The replica indices (= seeds) rank ``rank`` integrates."""
    if not 0 <= rank < world or per_gpu < 1:
        raise ValueError("rank must be in [0, world) and per_gpu >= 1")
    return [rank * per_gpu + r for r in range(per_gpu)]


class ThermoLog:
    """All-gathers the per-replica (E_pot, T) of every rank into ``frames`` [world*per_gpu, 2] fp64."""

    def __init__(self, per_gpu: int, device, group=None) -> None:
        self.per_gpu = int(per_gpu)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.local = torch.zeros(self.per_gpu, 2, dtype=torch.float64, device=device)
        self.parts = [torch.zeros_like(self.local) for _ in range(self.world)]
        self.frames: list[torch.Tensor] = []

    def gather(self, energies: torch.Tensor, temperatures: torch.Tensor) -> torch.Tensor:
        """One frame: this rank's values in, every rank's out (collective: every rank calls it)."""
        self.local[:, 0].copy_(energies.reshape(-1))
        self.local[:, 1].copy_(temperatures.reshape(-1))
        if self.world > 1:
            dist.all_gather(self.parts, self.local, group=self.group)
            frame = torch.cat(self.parts)
        else:
            frame = self.local.clone()
        return frame
