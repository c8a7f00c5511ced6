"""MatRIS bond graph: reverse-edge pairing and the line graph of ordered bond pairs.

The ragged builders of fastmd/graph/gpu_graph_builder.py: ``build_d2u`` restates ``_build_d2u`` (:217)
and ``build_line_graph`` ``_build_line_graph`` (:511), on ``fmd_reverse_pairs`` / ``fmd_line_graph``
(fastmd_b200/csrc/line_graph.cu). Like the reference's ragged path they read one count back to the
host (the undirected-edge count, the triplet count) to size their outputs; the triplet table grows
and is rebuilt when the first capacity guess overflows. CUDA tensors only.
"""
from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _lib
from ._lib import call, ptr, stream

_FLAG_TRIPLET_OVERFLOW = 128


def _workspace(name: str, *sizes, device) -> Tensor:
    nbytes = ctypes.c_size_t(0)
    call(name, *sizes, ctypes.byref(nbytes))
    return torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)


def build_d2u(center: Tensor, neighbor: Tensor, images: Tensor, n_atoms: int,
              presorted: bool = False) -> tuple[Tensor, Tensor]:
    """``(directed2undirected [E], undirected2directed [U])`` int32 of directed edges
    ``(center, neighbor, images)``; ``presorted``: the edges are in (centre, neighbour, image) order."""
    _lib.require_cuda(center, neighbor, images)
    dev = center.device
    E = center.shape[0]
    d2u = torch.empty(E, dtype=torch.int32, device=dev)
    u2d = torch.empty(E, dtype=torch.int32, device=dev)
    count = torch.zeros(1, dtype=torch.int64, device=dev)
    if E == 0:
        return d2u, u2d
    c, n = center.to(torch.int64).contiguous(), neighbor.to(torch.int64).contiguous()
    img = images.round().to(torch.int32).contiguous() if images.is_floating_point() else images.to(torch.int32)
    img = img.contiguous()
    ws = _workspace("fmd_reverse_pairs_workspace_bytes", E, device=dev)
    call("fmd_reverse_pairs", ptr(c), ptr(n), ptr(img), E, int(n_atoms), int(presorted), ptr(ws), ws.numel(),
         ptr(d2u), ptr(u2d), ptr(count), ptr(_lib.flags_word(dev)), stream(dev))
    return d2u, u2d[: int(count.item())]


def build_line_graph(center: Tensor, directed2undirected: Tensor, dist: Tensor, n_atoms: int, cutoff: float,
                     presorted: bool = False, capacity: int | None = None) -> Tensor:
    """Ordered triplets ``[T, 5]`` int32 ``[atom, u1, e1, u2, e2]`` over the edges shorter than ``cutoff``."""
    _lib.require_cuda(center, directed2undirected, dist)
    dev = center.device
    E = center.shape[0]
    if E == 0:
        return torch.empty((0, 5), dtype=torch.int32, device=dev)
    c = center.to(torch.int64).contiguous()
    d = dist.to(torch.float32).contiguous()
    d2u = directed2undirected.to(torch.int32).contiguous()
    ws = _workspace("fmd_line_graph_workspace_bytes", E, int(n_atoms), device=dev)
    count = torch.zeros(1, dtype=torch.int64, device=dev)
    cap = int(capacity) if capacity is not None else max(16 * E, 1024)
    while True:
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        out = torch.empty((cap, 5), dtype=torch.int32, device=dev)
        call("fmd_line_graph", ptr(c), ptr(d), ptr(d2u), E, int(n_atoms), float(cutoff), int(presorted), cap,
             ptr(ws), ws.numel(), ptr(out), ptr(count), ptr(flags), stream(dev))
        total = int(count.item())
        if total <= cap:
            if int(flags.item()) & ~_FLAG_TRIPLET_OVERFLOW:
                raise _lib.FastMDLibraryError(f"line graph: flags {int(flags.item())} (index out of range)")
            return out[:total]
        cap = total
