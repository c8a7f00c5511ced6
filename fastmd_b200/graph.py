"""Neighbour-list builders (the ``fastmd.graph`` surface) on libfastmd_b200 kernels.

* ``FixedCapacityGraphBuilder`` -- the capture-safe builder of
  fastmd/graph/fixed_capacity_builder.py:1030: a skin candidate list refreshed
  rarely (``refresh_candidates``, :1675) and an exact per-step re-filter into
  persistent padded buffers (``build``, :2181), published as a ``GraphBatch``.
  Edges only (the MACE / energy-tap topology, ``line_graph_cutoff=None``), or
  with the MatRIS bond graph (``line_graph_cutoff`` and ``t_capacity``): the
  undirected pairs and the triplets of short edges at fixed capacities, padded
  with sink atoms (``n_dummy`` sink rows) or far self-loops, on the all-padding
  topology after an overflow (``fmd_bond_graph``). R replicas of one system
  form a disjoint union (``replicas=R``; replica_batch.py:126).
* ``TensorGraphBuilder`` / ``neighbor_list`` -- the ragged eager path
  (gpu_graph_builder.py:935 / :108).

Differences from the reference by design: the candidate rows are sorted once
per refresh, so the per-step edges come out in canonical (centre, neighbour,
image) order without a per-step sort; the build also publishes the receiver
and sender CSRs the message-passing kernels read. Status values are device
tensors; nothing synchronises with the host inside ``build``.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from fastmd_b200 import _lib
from fastmd_b200._lib import call, ptr, stream

FLAG_INDEX_RANGE = 1
FLAG_EDGE_OVERFLOW = 2
FLAG_CANDIDATE_OVERFLOW = 4
FLAG_SKIN = 8
FLAG_NONFINITE = 16
FLAG_TRIPLET_OVERFLOW = 128
FLAG_INVALID_PAIRS = 256
_INVALID = (FLAG_EDGE_OVERFLOW | FLAG_CANDIDATE_OVERFLOW | FLAG_SKIN | FLAG_NONFINITE | FLAG_TRIPLET_OVERFLOW
            | FLAG_INVALID_PAIRS)


class NeighborOverflowError(RuntimeError):
    """A candidate row of the neighbour list was truncated (neighbor_list_backend.py)."""


@dataclass(frozen=True)
class PaddingRule:
    """The form of padded edge rows (fastmd/adapters/protocol.py:69): ``far_self_loops`` (a loop of a
    real atom, round robin, with an integer image at least twice the cutoff long: zero contribution
    under an exact radial cutoff, never a zero length), ``sink_atoms`` (loops of ``n_dummy`` sink rows,
    builds with a line graph) or ``exact_rc_loops`` (a loop of a real atom with image 0 whose edge vector
    the model takes from ``GraphBatch.edge_vec_override``: ``pad_vector``, by default ``(cutoff, 0, 0)``,
    exactly at the cutoff)."""

    kind: str = "far_self_loops"
    min_length: float = 0.0
    pad_vector: tuple | None = None

    def __post_init__(self):
        if self.kind not in ("far_self_loops", "sink_atoms", "exact_rc_loops"):
            raise ValueError(f"unknown kind {self.kind!r}")
        if not (self.min_length >= 0.0 and math.isfinite(self.min_length)):
            raise ValueError("min_length must be finite and >= 0")
        if self.min_length and self.kind != "far_self_loops":
            raise ValueError("min_length applies to far_self_loops only")
        if self.pad_vector is not None:
            if self.kind != "exact_rc_loops":
                raise ValueError("pad_vector applies to exact_rc_loops only")
            if len(self.pad_vector) != 3 or not all(math.isfinite(float(v)) for v in self.pad_vector):
                raise ValueError("pad_vector must be three finite numbers")


def exact_rc_pad_vector(padding: PaddingRule, cutoff: float) -> tuple[float, float, float]:
    """The padded rows' edge vector of ``exact_rc_loops`` (fixed_capacity_builder.py:1008-1014): the
    rule's ``pad_vector`` or ``(cutoff, 0, 0)``; its float32 length must not be inside the cutoff (nor 0)."""
    vector = tuple(float(v) for v in (padding.pad_vector or (cutoff, 0.0, 0.0)))
    length = float(np.linalg.norm(np.asarray(vector, np.float32)).astype(np.float32))
    if not length >= float(np.float32(cutoff)) or length == 0.0:
        raise ValueError(f"exact_rc_loops: pad_vector {vector} is shorter than the cutoff {cutoff}")
    return vector


@dataclass
class GraphBatch:
    """The published graph (protocol.py:144): real rows first, padding after ``n_edges``."""

    positions: Tensor        # [N, 3] wrapped float32
    cell: Tensor             # [3, 3] float32
    species: Tensor          # [N] int32 atomic numbers
    n_real: int
    edge_index: Tensor       # [E_cap, 2] int32 (centre, neighbour)
    edge_image: Tensor       # [E_cap, 3] float32
    n_edges: Tensor          # [1] int64
    cutoff: float
    padding: PaddingRule | None
    recv_off: Tensor | None = None   # [N + 1] int64 receiver (centre) CSR of the real edges
    send_off: Tensor | None = None   # [N + 1] int64 sender (neighbour) CSR
    send_perm: Tensor | None = None  # [E_cap] int32 edge ids grouped by sender
    replicas: int = 1
    element: Tensor | None = None    # model element rows (set by a model's prepare)
    element64: Tensor | None = None
    edge_vec_override: Tensor | None = None    # [E_cap, 3] float32: exact_rc_loops padded rows' vector, else 0
    directed2undirected: Tensor | None = None  # [E_cap] int32 (a builder with a line graph)
    undirected2directed: Tensor | None = None  # [U_cap] int32
    line_graph: Tensor | None = None           # [T_cap, 5] int32 [atom, u1, e1, u2, e2]

    @property
    def edge_dst(self) -> Tensor:
        return self.edge_index[:, 0]

    @property
    def edge_src(self) -> Tensor:
        return self.edge_index[:, 1]


class FixedCapacityGraphStatus:
    """Device-side status of one build (fixed_capacity_builder.py:757); the fields are
    derived from the build's FMD_FLAG_* word when read."""

    def __init__(self, flags: Tensor, n_edges: Tensor, max_displacement: Tensor, recv_off: Tensor,
                 n_real: int, n_triplets: Tensor | None = None) -> None:
        self.flags = flags
        self.edge_count = n_edges
        self.max_displacement = max_displacement
        self._recv_off = recv_off
        self._n_real = n_real
        self._n_triplets = n_triplets

    @property
    def overflow(self) -> Tensor:
        return (self.flags & _INVALID) != 0

    @property
    def candidate_valid(self) -> Tensor:
        return (self.flags & (FLAG_SKIN | FLAG_CANDIDATE_OVERFLOW | FLAG_NONFINITE)) == 0

    @property
    def candidate_capacity_valid(self) -> Tensor:
        return (self.flags & FLAG_CANDIDATE_OVERFLOW) == 0

    @property
    def invalid_pairs(self) -> Tensor:
        return (self.flags & FLAG_INVALID_PAIRS) != 0

    @property
    def undirected_count(self) -> Tensor:
        return self.edge_count // 2

    @property
    def triplet_count(self) -> Tensor:
        """Triplets of the stored rows (after an edge overflow: of the rows that fit)."""
        if self._n_triplets is None:
            return torch.zeros(1, dtype=torch.int64, device=self.flags.device)
        return self._n_triplets

    @property
    def isolated_atom_count(self) -> Tensor:
        degree = self._recv_off[1:self._n_real + 1] - self._recv_off[:self._n_real]
        return (degree == 0).sum().reshape(1)


def fixed_capacity_exceeded(status: FixedCapacityGraphStatus, builder) -> Tensor:
    """Device predicate: the real graph does not fit the builder (fixed_capacity_builder.py:796).
    Edges only: more edges than the edge capacity. With a line graph the padded triplets need a
    padded pair, so an edge count equal to the capacity overflows too, as do more triplets than
    the triplet capacity and invalid pairs."""
    if getattr(builder, "edges_only", True):
        return (status.edge_count[0] > builder.e_capacity) | ((status.flags[0] & FLAG_EDGE_OVERFLOW) != 0)
    return ((status.edge_count[0] >= builder.e_capacity) | (status.triplet_count[0] > builder.t_capacity)
            | status.invalid_pairs[0])


def estimate_max_neighbors(cutoff: float, atomic_density: float = 0.35, safety_factor: float = 5.0) -> int:
    """Per-atom candidate slots (neighbor_list_backend.py:77): safety * density * 4/3 pi rc^3,
    rounded up to a multiple of 16."""
    if cutoff <= 0:
        return 0
    expected = max(1, safety_factor * atomic_density * (4.0 / 3.0) * math.pi * cutoff**3)
    return int(math.ceil(expected / 16)) * 16


def self_loop_image(cell: Tensor, cutoff: float, min_length: float = 0.0) -> tuple[tuple[int, int, int], float]:
    """Far self-loop padding (fixed_capacity_builder.py:1006-1027): a whole number of the
    longest lattice vector, at least ``min_length`` and twice the cutoff."""
    lengths = cell.detach().cpu().double().norm(dim=1)
    axis = int(torch.argmax(lengths))
    longest = float(lengths[axis])
    if not longest > 0.0:
        raise ValueError("far self-loop padding needs a cell with a nonzero lattice vector")
    multiple = max(1, math.ceil(max(min_length, 2.0 * cutoff) / longest))
    image = [0, 0, 0]
    image[axis] = multiple
    return (image[0], image[1], image[2]), multiple * longest


def _host_cell(cell: Tensor):
    arr = np.ascontiguousarray(cell.detach().cpu().numpy().astype(np.float32).reshape(9))
    return arr, arr.ctypes.data_as(ctypes.c_void_p)


class FixedCapacityGraphBuilder:
    """Capture-safe graph builder with static shapes (fixed_capacity_builder.py:1030).

    ``u_capacity`` undirected pairs (``e_capacity = 2 u_capacity`` directed rows) over the whole
    union of ``replicas`` copies of the system. ``candidate_cutoff`` (default ``cutoff + 1e-6``)
    sets the skin: a step stays exact while no atom moved more than half the skin since the
    last ``refresh_candidates``. With ``line_graph_cutoff`` (at most the atom cutoff) and
    ``t_capacity`` the build also publishes the MatRIS bond graph (``directed2undirected``,
    ``undirected2directed``, ``line_graph`` on the batch); its padding is ``sink_atoms`` (the
    default then: ``n_dummy`` sink rows after the real atoms, positions at the origin, species 1)
    or ``far_self_loops``.
    """

    def __init__(self, *, cell: Tensor, atomic_numbers: Tensor, u_capacity: int, t_capacity: int = 0,
                 pbc: Tensor | None = None, atom_graph_cutoff: float = 6.0, line_graph_cutoff: float | None = None,
                 n_dummy: int = 0, device="cuda", candidate_cutoff: float | None = None,
                 padding: PaddingRule | None = None, replicas: int = 1, max_neighbors: int | None = None,
                 minimum_image: bool = False, candidates_from: "FixedCapacityGraphBuilder | None" = None,
                 positions_dtype: torch.dtype = torch.float32, **unused) -> None:
        self.edges_only = line_graph_cutoff is None
        if pbc is not None and not bool(torch.as_tensor(pbc).all()):
            raise ValueError("this build implements fully periodic cells")
        if self.edges_only:
            padding = PaddingRule("far_self_loops") if padding is None else padding
            if padding.kind not in ("far_self_loops", "exact_rc_loops"):
                raise ValueError("edges-only builds pad with far self-loops or exact-rc loops here")
            if int(u_capacity) <= 0 or t_capacity != 0:
                raise ValueError("an edges-only builder needs u_capacity > 0 and t_capacity == 0")
        else:
            padding = PaddingRule("sink_atoms") if padding is None else padding
            if int(u_capacity) <= 0 or int(t_capacity) <= 0 or (padding.kind == "sink_atoms" and int(n_dummy) <= 0):
                raise ValueError("capacities and n_dummy must be positive")
            if float(line_graph_cutoff) > float(atom_graph_cutoff):
                raise ValueError("line graph cutoff must not exceed atom graph cutoff")
            if padding.kind not in ("sink_atoms", "far_self_loops"):
                raise ValueError("a builder with a line graph pads with sink atoms or far self-loops")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise _lib.FastMDLibraryError("the graph builders run on CUDA devices only")
        if positions_dtype not in (torch.float32, torch.float64):
            raise ValueError(f"positions_dtype must be float32 or float64, got {positions_dtype}")
        self.positions_dtype = positions_dtype
        self.minimum_image = bool(minimum_image)
        self.padding = padding
        self.cell = cell.detach().to(device=self.device, dtype=torch.float32).reshape(3, 3).contiguous()
        self._cell_host, self._cell_ptr = _host_cell(self.cell)
        self.replicas = int(replicas)
        species = torch.as_tensor(atomic_numbers).to(device=self.device, dtype=torch.int32).reshape(-1)
        self.n_atoms = int(species.shape[0])  # per replica
        self.n_real = self.n_atoms * self.replicas
        self.u_capacity = int(u_capacity)
        self.e_capacity = 2 * self.u_capacity
        self.t_capacity = 0 if self.edges_only else int(t_capacity)
        self.n_dummy = int(n_dummy) if padding.kind == "sink_atoms" else 0
        self.atom_graph_cutoff = float(atom_graph_cutoff)
        self.line_graph_cutoff = None if self.edges_only else float(line_graph_cutoff)
        self.candidate_cutoff = float(candidate_cutoff or (self.atom_graph_cutoff + 1.0e-6))
        self.skin = self.candidate_cutoff - self.atom_graph_cutoff
        self.buffer_max = int(max_neighbors or estimate_max_neighbors(self.candidate_cutoff, safety_factor=2.0))
        if padding.kind == "exact_rc_loops":  # loops with image 0, the edge vector overridden
            self.pad_vector = exact_rc_pad_vector(padding, self.atom_graph_cutoff)
            image, length = (0, 0, 0), float(np.linalg.norm(self.pad_vector))
            self._pad_vector_host = (ctypes.c_float * 3)(*self.pad_vector)
        else:
            image, length = self_loop_image(self.cell, self.atom_graph_cutoff, padding.min_length)
        self.pad_image = image
        self.pad_length = length
        self._pad_image_host = (ctypes.c_int32 * 3)(*image)  # sink padding: the bond graph rewrites the loops
        N, B, E, dev = self.n_real, self.buffer_max, self.e_capacity, self.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.cand_nbr = torch.full((N, B), N, **i32)
        self.cand_shift = torch.zeros((N, B, 3), **i32)
        self.cand_count = torch.zeros(N, **i32)
        self.reference_positions = torch.zeros(N, 3, dtype=torch.float32, device=dev)
        self.reference_wraps = torch.zeros(N, 3, **i32)
        self.wrap_delta = torch.zeros(N, 3, **i32)
        self.refresh_flags = torch.zeros(1, **i32)
        self.flags = torch.zeros(1, **i32)
        self.max_displacement = torch.zeros(self.replicas, dtype=torch.float32, device=dev)
        nbytes = ctypes.c_size_t(0)
        call("fmd_cell_list_workspace_bytes", self._cell_ptr, self.candidate_cutoff, self.n_atoms, self.replicas,
             ctypes.byref(nbytes))
        self._cell_ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
        call("fmd_refilter_workspace_bytes", self.n_atoms, self.replicas, ctypes.byref(nbytes))
        self._refilter_ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
        self.positions32 = torch.zeros(N, 3, dtype=torch.float32, device=dev)
        rows = N + self.n_dummy  # sink rows after the real atoms (at the origin, species 1)
        # float64 positions (fixed_capacity_builder.py:2315): the edges come from the float32 wrap of the
        # rounded coordinates; the published positions are the float64 coordinates minus the same whole
        # lattice vectors of the float64 cell (the caller's cell in float64)
        self.float64 = positions_dtype == torch.float64
        if self.float64:
            cell64 = cell.detach().to(dtype=torch.float64).reshape(3, 3)
            self._cell64_host = np.ascontiguousarray(cell64.cpu().numpy().reshape(9))
            self._cell64_ptr = self._cell64_host.ctypes.data_as(ctypes.c_void_p)
            self.wrapped32 = torch.zeros(N, 3, dtype=torch.float32, device=dev)
            self._positions64 = torch.zeros(N, 3, dtype=torch.float64, device=dev)
        self.batch = GraphBatch(
            positions=torch.zeros(rows, 3, dtype=positions_dtype, device=dev),
            cell=cell64.to(dev).contiguous() if self.float64 else self.cell,
            species=torch.cat([species.repeat(self.replicas), torch.ones(self.n_dummy, **i32)]),
            n_real=N,
            edge_index=torch.zeros(E, 2, **i32),
            edge_image=torch.zeros(E, 3, dtype=torch.float32, device=dev),
            n_edges=torch.zeros(1, dtype=torch.int64, device=dev),
            cutoff=self.atom_graph_cutoff,
            padding=padding,
            recv_off=torch.zeros(N + 1, dtype=torch.int64, device=dev),
            send_off=torch.zeros(N + 1, dtype=torch.int64, device=dev),
            send_perm=torch.zeros(E, **i32),
            replicas=self.replicas,
        )
        if padding.kind == "exact_rc_loops":
            self.batch.edge_vec_override = torch.zeros(E, 3, dtype=torch.float32, device=dev)
        self.n_triplets = None
        if not self.edges_only:
            U, T = self.u_capacity, self.t_capacity
            self.batch.directed2undirected = torch.zeros(E, **i32)
            self.batch.undirected2directed = torch.zeros(U, **i32)
            self.batch.line_graph = torch.zeros((T, 5), **i32)
            self.n_triplets = torch.zeros(1, dtype=torch.int64, device=dev)
            call("fmd_bond_graph_workspace_bytes", N, E, ctypes.byref(nbytes))
            self._bond_ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
            self._bond_pad_image = (ctypes.c_int32 * 3)(*image)
        self._candidate_initialized = False
        self._candidate_owner = self
        if candidates_from is not None:
            self._share_candidates(candidates_from)

    # the candidate state a ``candidates_from`` builder reads from its owner (fixed_capacity_builder.py:666)
    _CANDIDATE_STATE = ("cand_nbr", "cand_shift", "cand_count", "reference_positions", "reference_wraps",
                        "wrap_delta", "refresh_flags")

    def _share_candidates(self, owner: "FixedCapacityGraphBuilder") -> None:
        """Read ``owner``'s candidate list (its refreshes are this builder's): same atoms, cell,
        candidate cutoff and slot count required."""
        owner = owner._candidate_owner
        if (owner.n_real != self.n_real or owner.buffer_max != self.buffer_max
                or owner.candidate_cutoff != self.candidate_cutoff or not torch.equal(owner.cell, self.cell)
                or owner.replicas != self.replicas or owner.minimum_image != self.minimum_image):
            raise ValueError("candidates_from: the owner builds another system, cutoff or slot count")
        for name in self._CANDIDATE_STATE:
            setattr(self, name, getattr(owner, name))
        self._candidate_owner = owner

    def resized(self, u_capacity: int, t_capacity: int | None = None) -> "FixedCapacityGraphBuilder":
        """A builder of the same system with other capacities (new buffers; the candidates
        are refreshed by the caller)."""
        return FixedCapacityGraphBuilder(
            cell=self.cell, atomic_numbers=self.batch.species[:self.n_atoms], u_capacity=u_capacity,
            t_capacity=self.t_capacity if t_capacity is None else t_capacity,
            atom_graph_cutoff=self.atom_graph_cutoff, line_graph_cutoff=self.line_graph_cutoff,
            n_dummy=self.n_dummy, device=self.device, candidate_cutoff=self.candidate_cutoff,
            padding=self.padding, replicas=self.replicas, max_neighbors=self.buffer_max,
            minimum_image=self.minimum_image, positions_dtype=self.positions_dtype)

    # ------------------------------------------------------------------ inputs
    def _positions(self, positions: Tensor) -> Tensor:
        if positions.shape != (self.n_real, 3):
            raise ValueError(f"positions must have shape {(self.n_real, 3)}, got {tuple(positions.shape)}")
        if positions.dtype == torch.float32 and positions.is_contiguous() and positions.device == self.device:
            return positions
        self.positions32.copy_(positions)
        return self.positions32

    # ------------------------------------------------------------- candidates
    @torch.no_grad()
    def refresh_candidates(self, positions: Tensor) -> None:
        """The skin candidate list of the current positions and the refresh snapshot
        (fixed_capacity_builder.py:1675); stream ordered, no host synchronisation."""
        pos = self._positions(positions)
        self.refresh_flags.zero_()
        call("fmd_candidates_build", ptr(pos), self._cell_ptr, self.n_atoms, self.replicas, self.candidate_cutoff,
             self.buffer_max, ptr(self.cand_nbr), ptr(self.cand_shift), ptr(self.cand_count),
             ptr(self.reference_positions), ptr(self.reference_wraps), ptr(self.wrap_delta), ptr(self._cell_ws),
             self._cell_ws.numel(), ptr(self.refresh_flags), stream(self.device))
        self._candidate_owner._candidate_initialized = True

    def assert_candidate_capacity(self) -> None:
        """Raise on the slow path if a candidate row was truncated (host read)."""
        if int(self.refresh_flags.item()) & FLAG_CANDIDATE_OVERFLOW:
            raise NeighborOverflowError(
                f"more than {self.buffer_max} candidates for an atom (max {int(self.cand_count.max())})")

    # ------------------------------------------------------------------ build
    @torch.no_grad()
    def build(self, positions: Tensor, *, rebuild_candidates: bool = True, predicate=None,
              flags: Tensor | None = None) -> tuple[GraphBatch, FixedCapacityGraphStatus]:
        """Edges of ``positions`` into the persistent buffers; returns ``(batch, status)``
        (fixed_capacity_builder.py:2181). ``flags``: an int32 word the build ORs its
        FMD_FLAG_* bits into (a whole-step window's); default the builder's own, reset here."""
        if predicate is not None:
            raise ValueError("a caller's edge predicate needs the ghost-row builder (not in this build)")
        pos = self._positions(positions)
        if rebuild_candidates:
            self.refresh_candidates(pos)
        elif not self._candidate_owner._candidate_initialized:
            raise RuntimeError("refresh_candidates must run before candidate reuse")
        if flags is None:
            flags = self.flags
            flags.copy_(self.refresh_flags)
        wrapped = self.wrapped32 if self.float64 else self.batch.positions
        call("fmd_refilter_edges", ptr(pos), self._cell_ptr, self.n_atoms, self.replicas,
             ptr(self.reference_positions), ptr(self.reference_wraps), ptr(self.cand_nbr), ptr(self.cand_shift),
             ptr(self.cand_count), self.buffer_max, self.atom_graph_cutoff, self.skin, self.e_capacity,
             self._pad_image_host, int(self.minimum_image), ptr(wrapped), ptr(self.wrap_delta),
             ptr(self.batch.edge_index), ptr(self.batch.edge_image), ptr(self.batch.recv_off), ptr(self.batch.send_off),
             ptr(self.batch.send_perm), ptr(self.batch.n_edges), ptr(self.max_displacement), ptr(self._refilter_ws),
             self._refilter_ws.numel(), ptr(flags), stream(self.device))
        if self.padding.kind == "exact_rc_loops":
            call("fmd_pad_vector_override", ptr(self.batch.n_edges), self.e_capacity, self._pad_vector_host,
                 ptr(self.batch.edge_vec_override), stream(self.device))
        if self.float64:
            p64 = positions
            if not (p64.dtype == torch.float64 and p64.is_contiguous() and p64.device == self.device):
                p64 = self._positions64
                p64.copy_(positions)
            call("fmd_model_positions_f64", ptr(p64), self.n_real, self._cell_ptr, self._cell64_ptr,
                 ptr(self.batch.positions), stream(self.device))
        if not self.edges_only:
            b = self.batch
            call("fmd_bond_graph", ptr(wrapped), self._cell_ptr, self.n_real, ptr(b.edge_index), ptr(b.edge_image),
                 ptr(b.n_edges), self.u_capacity, self.t_capacity, self.line_graph_cutoff,
                 0 if self.padding.kind == "sink_atoms" else 1, self.n_dummy, self._bond_pad_image, ptr(self._bond_ws),
                 self._bond_ws.numel(), ptr(b.directed2undirected), ptr(b.undirected2directed), ptr(b.line_graph),
                 ptr(self.n_triplets), ptr(flags), stream(self.device))
        status = FixedCapacityGraphStatus(flags, self.batch.n_edges, self.max_displacement, self.batch.recv_off,
                                          self.n_real, self.n_triplets)
        return self.batch, status


def _grown(current: int, needed: int) -> int:
    return int(math.ceil(max(needed, 2 * current) / 16)) * 16


@torch.no_grad()
def neighbor_list(positions: Tensor, cell: Tensor, cutoff: float, *, max_neighbors: int | None = None,
                  return_wrapped: bool = False):
    """Full neighbour list sorted by (centre, neighbour, image) of one periodic system
    (gpu_graph_builder.py:108): ``(center, neighbor, images, dist)`` (int64, int64, int32 [E, 3],
    float32), from candidates at ``cutoff + 1e-6`` kept when ``|(x_j - x_i) + image @ cell| < cutoff``.
    Eager: one host read of the edge count (and a rerun when a candidate row or the edge
    buffer was too small)."""
    _lib.require_cuda(positions)
    dev = positions.device
    pos = positions.detach().to(torch.float32).contiguous()
    n = pos.shape[0]
    cell_t = cell.detach().reshape(3, 3)
    cell_host, cell_ptr = _host_cell(cell_t)
    volume = abs(float(np.linalg.det(cell_host.reshape(3, 3).astype(np.float64))))
    density = n / max(volume, 1e-9)
    bmax = int(max_neighbors or estimate_max_neighbors(cutoff, atomic_density=max(density, 1e-3), safety_factor=2.0))
    e_cap = int(n * max(16, bmax // 2))
    while True:
        nbytes = ctypes.c_size_t(0)
        call("fmd_neighbor_list_workspace_bytes", cell_ptr, float(cutoff), n, bmax, ctypes.byref(nbytes))
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
        center = torch.empty(e_cap, dtype=torch.int64, device=dev)
        neighbor = torch.empty(e_cap, dtype=torch.int64, device=dev)
        images = torch.empty(e_cap, 3, dtype=torch.int32, device=dev)
        dist = torch.empty(e_cap, dtype=torch.float32, device=dev)
        offsets = torch.empty(n + 1, dtype=torch.int64, device=dev)
        wrapped = torch.empty(n, 3, dtype=torch.float32, device=dev)
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        call("fmd_neighbor_list", ptr(pos), cell_ptr, n, float(cutoff), bmax, e_cap, ptr(wrapped), ptr(center),
             ptr(neighbor), ptr(images), ptr(dist), ptr(offsets), ptr(ws), ws.numel(), ptr(flags), stream(dev))
        total, flag = (int(v) for v in torch.stack([offsets[n], flags[0].long()]).tolist())
        if flag & FLAG_CANDIDATE_OVERFLOW:
            bmax = _grown(bmax, bmax + 1)
            continue
        if total > e_cap:
            e_cap = total
            continue
        out = (center[:total], neighbor[:total], images[:total], dist[:total])
        return (*out, wrapped, offsets) if return_wrapped else out


class TensorGraphBuilder:
    """Ragged (eager) edges-only builder (gpu_graph_builder.py:935): ``build(positions)``
    returns a ``GraphBatch`` of exactly the real edges (no padding)."""

    def __init__(self, *, cell: Tensor, atomic_numbers: Tensor, atom_graph_cutoff: float = 6.0,
                 line_graph_cutoff: float | None = None, device="cuda", max_neighbors: int | None = None,
                 **unused) -> None:
        if line_graph_cutoff is not None:
            raise ValueError("this build implements the edges-only ragged builder")
        self.device = torch.device(device)
        self.cell = cell.detach().to(device=self.device, dtype=torch.float32).reshape(3, 3).contiguous()
        self.atomic_numbers = torch.as_tensor(atomic_numbers).to(device=self.device, dtype=torch.int32)
        self.n_atoms = int(self.atomic_numbers.shape[0])
        self.atom_graph_cutoff = float(atom_graph_cutoff)
        self.max_neighbors = max_neighbors

    @torch.no_grad()
    def build(self, positions: Tensor) -> GraphBatch:
        center, neighbor, images, _, wrapped, offsets = neighbor_list(
            positions.to(self.device), self.cell, self.atom_graph_cutoff, max_neighbors=self.max_neighbors,
            return_wrapped=True)
        from fastmd_b200.ops import segment_csr

        perm, send_off = segment_csr(neighbor, self.n_atoms)
        return GraphBatch(
            positions=wrapped, cell=self.cell, species=self.atomic_numbers, n_real=self.n_atoms,
            edge_index=torch.stack([center, neighbor], dim=1).to(torch.int32).contiguous(),
            edge_image=images.to(torch.float32).contiguous(),
            n_edges=torch.full((1,), center.shape[0], dtype=torch.int64, device=self.device),
            cutoff=self.atom_graph_cutoff, padding=None, recv_off=offsets, send_off=send_off,
            send_perm=perm.to(torch.int32))

    __call__ = build
