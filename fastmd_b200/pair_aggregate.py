"""Directed-edge <-> undirected-pair aggregation of the MatRIS atom graph.

The operator surface of fastmd/models/matris/op/triton_directed_pair_aggregate.py:
``directed_pair_average`` (:311) averages the two directed rows of every undirected pair,
``undirected_pair_expand`` (:328) copies each pair row back onto both directed rows, both
differentiable, and ``pair_index_bijection_reason`` (:261) is the host-side admission check of the
``pair_index [U, 2]`` bijection. The four maps run in ``fmd_pair_aggregate``
(fastmd_b200/csrc/pair_aggregate.cu), bit-identical to the reference's kernels. Inputs keep their row
stride (``packed[:, :D]`` is read in place; only ``stride(1) != 1`` is copied), outputs are fresh
contiguous tensors. Shape errors raise ``ValueError`` with the reference's messages; where the
reference falls back to torch (CPU tensors) this build raises, there is no CPU path.
"""
from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd import Function

from . import _lib
from ._lib import FastMDLibraryError, call, ptr, stream

AVERAGE, AVERAGE_BWD, EXPAND, EXPAND_BWD = 0, 1, 2, 3


def _run(op: int, src: Tensor, pair_index: Tensor, rows_out: int) -> Tensor:
    dim = src.shape[1]
    out = torch.empty((rows_out, dim), device=src.device, dtype=torch.float32)
    call("fmd_pair_aggregate", op, ptr(src), src.stride(0), ptr(pair_index), pair_index.shape[0], dim, ptr(out),
         ptr(_lib.flags_word(src.device)), stream(src.device))
    return out


def _rows(t: Tensor) -> Tensor:
    """``t`` with unit column stride (its row stride kept)."""
    return t if t.stride(1) == 1 and t.stride(0) >= max(t.shape[1], 1) else t.contiguous()


class _DirectedPairAverage(Function):
    @staticmethod
    def forward(ctx, data, pair_index):
        ctx.save_for_backward(pair_index)
        ctx.num_directed = data.shape[0]
        return _run(AVERAGE, _rows(data), pair_index, pair_index.shape[0])

    @staticmethod
    def backward(ctx, gout):
        (pair_index,) = ctx.saved_tensors
        return _run(AVERAGE_BWD, _rows(gout), pair_index, ctx.num_directed), None


class _UndirectedPairExpand(Function):
    @staticmethod
    def forward(ctx, data, pair_index, num_directed):
        ctx.save_for_backward(pair_index)
        return _run(EXPAND, _rows(data), pair_index, num_directed)

    @staticmethod
    def backward(ctx, gout):
        (pair_index,) = ctx.saved_tensors
        return _run(EXPAND_BWD, _rows(gout), pair_index, pair_index.shape[0]), None, None


def pair_index_bijection_reason(pair_index, num_directed) -> str | None:
    """Why ``pair_index`` is not a pair bijection onto ``num_directed`` rows, else None.

    The checks and reasons of the reference's admission check (triton_directed_pair_aggregate.py:261):
    an integer ``[U, 2]`` tensor, ``num_directed == 2U``, every value in range, no directed row twice.
    It reads index values (a device sync for CUDA tensors): admission and tests, never the hot path.
    """
    if not isinstance(pair_index, torch.Tensor):
        return "not_tensor"
    if pair_index.dim() != 2 or pair_index.shape[1] != 2:
        return f"pair_index_shape: expected [U, 2], got {list(pair_index.shape)}"
    if pair_index.dtype not in (torch.int32, torch.int64):
        return f"index_dtype: {pair_index.dtype}"
    num_directed = int(num_directed)
    num_pairs = pair_index.shape[0]
    if num_directed != 2 * num_pairs:
        return f"num_directed: {num_directed} != 2U = {2 * num_pairs}"
    if num_pairs == 0:
        return None
    flat = pair_index.reshape(-1).long()
    low, high = (int(v) for v in torch.stack((flat.min(), flat.max())).tolist())
    if low < 0 or high >= num_directed:
        return f"index_out_of_range: [{low}, {high}] not within [0, {num_directed})"
    if bool((torch.bincount(flat, minlength=num_directed) != 1).any()):
        return "duplicate_directed_row"
    return None


def _shape_error(data: Tensor, pair_index: Tensor, num_directed: int | None, what: str) -> ValueError:
    if data.dim() != 2 or pair_index.dim() != 2 or pair_index.shape[1] != 2:
        return ValueError(f"{what}: expected data [rows, D] and pair_index [U, 2], "
                          f"got {tuple(data.shape)}, {tuple(pair_index.shape)}")
    u = pair_index.shape[0]
    if num_directed is not None and num_directed != 2 * u:
        return ValueError(f"{what}: num_directed must be 2U (a pair bijection); "
                          f"got num_directed = {num_directed} for U = {u}")
    per_pair = 1 if num_directed is not None else 2
    return ValueError(f"{what}: expected {per_pair} data row(s) per pair (E == 2U directed rows), "
                      f"got {data.shape[0]} rows for U = {u}")


def _prepare(data: Tensor, pair_index: Tensor) -> Tensor:
    _lib.require_cuda(data, pair_index)
    if data.dtype != torch.float32:
        raise FastMDLibraryError(f"pair aggregation: float32 data only, got {data.dtype}")
    if pair_index.dtype not in (torch.int32, torch.int64):
        raise FastMDLibraryError(f"pair aggregation: int32/int64 pair_index only, got {pair_index.dtype}")
    return pair_index.to(torch.int64).contiguous()


def directed_pair_average(data: Tensor, pair_index: Tensor) -> Tensor:
    """``(data[pair_index[:, 0]] + data[pair_index[:, 1]]) / 2`` for data ``[2U, D]``."""
    ds, ps = data.shape, pair_index.shape
    if len(ds) != 2 or len(ps) != 2 or ps[1] != 2 or ds[0] != 2 * ps[0]:
        raise _shape_error(data, pair_index, None, "directed_pair_average")
    return _DirectedPairAverage.apply(data, _prepare(data, pair_index))


def undirected_pair_expand(data: Tensor, pair_index: Tensor, num_directed: int) -> Tensor:
    """``out[pair_index[u, k]] = data[u]`` for data ``[U, D]``; ``num_directed`` must be 2U."""
    num_directed = int(num_directed)
    ds, ps = data.shape, pair_index.shape
    if len(ds) != 2 or len(ps) != 2 or ps[1] != 2 or ds[0] != ps[0] or num_directed != 2 * ps[0]:
        raise _shape_error(data, pair_index, num_directed, "undirected_pair_expand")
    return _UndirectedPairExpand.apply(data, _prepare(data, pair_index), num_directed)


__all__ = ["directed_pair_average", "undirected_pair_expand", "pair_index_bijection_reason"]
