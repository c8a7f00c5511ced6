"""The ``model_graph`` execution mode: one CUDA graph of the model's energy and forces per capacity bucket.

The runner of fastmd/execution/cuda_graph.py (``BucketedGraphRunner`` :449) for edges-only models. A
ragged build (``TensorGraphBuilder.build``: exactly the real edges) changes its edge count from step to
step; the runner copies it into the persistent padded batch of a capacity bucket (real rows first, then
far self-loop rows, as ``_PaddedEdgesWorkspace`` :209 writes them for a model whose padding rule is far
self-loops) and replays the CUDA graph of the model's fused energy/force evaluation captured for that
bucket. A bucket's pair capacity is ``tier(u, u_step, min_pad_u)`` (fastmd/engine/capacity_policy.py:19:
the next multiple of ``u_step`` above the pair count u, one more step when that leaves less than
``min_pad_u`` pairs of slack). Selection (cuda_graph.py:677 ``_select``): the smallest cached bucket
that holds the demand is replayed; a demand no cached bucket holds is captured into a new bucket (the
cached ones stay); a change of atom count drops every bucket and captures anew (a graph replays a fixed
atom count). Counts are host-known shapes: selection reads nothing from the device.

The padded rows add exactly nothing: the fused kernels visit only the real rows (the batch's device
count ``n_edges`` and its receiver/sender CSRs of the real edges), so a replay returns the same energies
and forces, bit for bit, as the eager evaluation of the ragged build. Outputs are the model's persistent
buffers, valid until the next ``run``.
"""
from __future__ import annotations


from dataclasses import dataclass

import torch

from fastmd_b200._capture import quiet_gc
from torch import Tensor

from .graph import GraphBatch, PaddingRule, self_loop_image


def tier(value: int, step: int, min_pad: int) -> int:
    """The capacity of one bucket: the next multiple of ``step`` above ``value``, one more step if that
    leaves less than ``min_pad`` slack (capacity_policy.py:19)."""
    capacity = (int(value) // step + 1) * step
    return capacity + step if capacity - int(value) < min_pad else capacity


def smallest_fitting_key(keys, u: int, u_step: int):
    """The smallest cached pair capacity strictly above the demand ``u`` (cuda_graph.py:435), or None."""
    fitting = [key for key in keys if key > u]
    return min(fitting, key=lambda key: ((key - u) / u_step, key)) if fitting else None


@dataclass
class _PaddedEdges:
    """The persistent batch of one bucket: ``e_max = 2 u_cap`` edge rows, the real rows of each update
    first, far self-loops after them (atom k mod n of padding row k, an integer image at least twice
    the cutoff long)."""

    batch: GraphBatch
    e_max: int
    loop_atoms: Tensor
    loop_image: Tensor
    row_ids: Tensor

    @classmethod
    def create(cls, sample: GraphBatch, u_cap: int) -> "_PaddedEdges":
        dev = sample.edge_index.device
        n, e_max = sample.n_real, 2 * int(u_cap)
        image, _ = self_loop_image(sample.cell, sample.cutoff)
        loop_atoms = (torch.arange(e_max, device=dev) % n).to(torch.int32)
        loop_image = torch.tensor(image, dtype=torch.float32, device=dev)
        batch = GraphBatch(
            positions=torch.zeros(n, 3, dtype=torch.float32, device=dev), cell=sample.cell.clone(),
            species=sample.species.clone(), n_real=n,
            edge_index=torch.zeros(e_max, 2, dtype=torch.int32, device=dev),
            edge_image=torch.zeros(e_max, 3, dtype=torch.float32, device=dev),
            n_edges=torch.zeros(1, dtype=torch.int64, device=dev), cutoff=sample.cutoff,
            padding=PaddingRule("far_self_loops"),
            recv_off=torch.zeros(n + 1, dtype=torch.int64, device=dev),
            send_off=torch.zeros(n + 1, dtype=torch.int64, device=dev),
            send_perm=torch.zeros(e_max, dtype=torch.int32, device=dev))
        return cls(batch, e_max, loop_atoms, loop_image, torch.arange(e_max, dtype=torch.int32, device=dev))

    @torch.no_grad()
    def update(self, g: GraphBatch) -> None:
        """Copy a ragged build of the same atoms into the padded batch (device copies, no sync)."""
        pb, e = self.batch, int(g.edge_index.shape[0])
        if g.n_real != pb.n_real or e > self.e_max:
            raise ValueError(f"a build of {g.n_real} atoms / {e} edges does not fit this bucket "
                             f"({pb.n_real} atoms / {self.e_max} edge rows)")
        pb.positions.copy_(g.positions)
        pb.cell.copy_(g.cell)
        pb.species.copy_(g.species)
        pb.edge_index[:e].copy_(g.edge_index)
        pb.edge_image[:e].copy_(g.edge_image)
        pb.n_edges.copy_(g.n_edges)
        pb.recv_off.copy_(g.recv_off)
        pb.send_off.copy_(g.send_off)
        pb.send_perm[:e].copy_(g.send_perm)
        if e < self.e_max:
            pb.edge_index[e:, 0].copy_(self.loop_atoms[: self.e_max - e])
            pb.edge_index[e:, 1].copy_(self.loop_atoms[: self.e_max - e])
            pb.edge_image[e:].copy_(self.loop_image.expand(self.e_max - e, 3))
            pb.send_perm[e:].copy_(self.row_ids[e:])


class BucketedGraphRunner:
    """Captures one CUDA graph per capacity bucket of a model's fused energy/force evaluation and
    replays the bucket that holds each build (cuda_graph.py:449). ``model``: an object with
    ``prepare(batch)`` and ``energy_forces_fused(batch, n_systems)`` (``MACEModel``). ``task``:
    ``"ef"`` or ``"e"`` (energies and forces are evaluated together either way)."""

    def __init__(self, model, task: str = "ef", u_step: int = 512, min_pad_u: int = 256, warmup: int = 3,
                 n_systems: int = 1) -> None:
        if task not in ("e", "ef"):
            raise ValueError(f"model_graph task {task!r}: this build captures energies and forces ('e', 'ef')")
        if u_step < 1 or min_pad_u < 0 or warmup < 1:
            raise ValueError("u_step >= 1, min_pad_u >= 0 and warmup >= 1")
        self.model = model
        self.task = task
        self.u_step, self.min_pad_u, self.warmup = int(u_step), int(min_pad_u), int(warmup)
        self.n_systems = int(n_systems)
        self.cache: dict[int, dict] = {}
        self.captures = 0
        self.warmup_runs = 0
        self.cache_fit_reuses = 0
        self.pool_resets = 0
        self._n_real: int | None = None
        self.pool = None

    # ------------------------------------------------------------------ selection
    def bucket_key(self, u: int) -> int:
        return tier(u, self.u_step, self.min_pad_u)

    def select(self, n: int, u: int) -> tuple[int, str | None]:
        """(pair capacity, action) for n atoms and u real pairs, without changing state: action None
        (replay), "capture" (a new bucket beside the cached ones) or "rebind" (another atom count:
        drop every bucket, then capture)."""
        requested = self.bucket_key(u)
        if self.cache and n != self._n_real:
            return requested, "rebind"
        key = smallest_fitting_key(self.cache.keys(), u, self.u_step)
        if key is not None:
            return key, None
        return requested, "capture"

    # ------------------------------------------------------------------ capture / replay
    def release(self) -> None:
        """Drop every captured bucket and its graph pool."""
        if self.cache:
            torch.cuda.synchronize()
        for ent in self.cache.values():
            ent["graph"].reset()
        self.cache.clear()
        self.pool = None
        self.pool_resets += 1

    def _capture(self, u_cap: int, sample: GraphBatch) -> dict:
        workspace = _PaddedEdges.create(sample, u_cap)
        workspace.update(sample)
        batch = self.model.prepare(workspace.batch)
        side = torch.cuda.Stream(device=batch.positions.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(self.warmup):  # buffers, weight copies and splits are made here, not in the capture
                self.model.energy_forces_fused(batch, n_systems=self.n_systems)
                self.warmup_runs += 1
        torch.cuda.current_stream().wait_stream(side)
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        with quiet_gc(), torch.cuda.graph(graph, pool=self.pool):
            energy, forces = self.model.energy_forces_fused(batch, n_systems=self.n_systems)
        self.captures += 1
        return {"graph": graph, "workspace": workspace, "energy": energy, "forces": forces, "u_cap": u_cap}

    def run(self, g: GraphBatch) -> tuple[Tensor, Tensor]:
        """(energies [n_systems] fp64, forces [N, 3] float32) of a ragged build, by replay of its bucket's
        graph (captured first on a miss). The tensors are the model's buffers, valid until the next run."""
        n, u = g.n_real, int(g.edge_index.shape[0]) // 2 + int(g.edge_index.shape[0]) % 2
        key, action = self.select(n, u)
        if action == "rebind":
            self.release()
        if action is not None:
            self.cache[key] = self._capture(key, g)
            self._n_real = n
        elif key != self.bucket_key(u):
            self.cache_fit_reuses += 1
        ent = self.cache[key]
        ent["workspace"].update(g)
        ent["graph"].replay()
        return ent["energy"], ent["forces"]

    def stats(self) -> dict[str, object]:
        return {"captures": self.captures, "warmup_runs": self.warmup_runs, "cache_fit_reuses": self.cache_fit_reuses,
                "pool_resets": self.pool_resets, "cached_buckets": sorted(self.cache)}


__all__ = ["BucketedGraphRunner", "smallest_fitting_key", "tier"]
