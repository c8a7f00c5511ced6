"""Edge/node operators of the message-passing hot path (the ``fastmd.ops`` surface).

Drop-in for the reference operators, same names, argument meaning and errors:

* ``aligned_gather_cat3`` / ``aligned_gather_cat4``
  (fastmd/models/matris/op/triton_gather_cat.py:181 / :353);
* ``gather_cat``: the mixed-width form (the reference falls back to ``torch.cat``
  for parts of different widths, triton_gather_cat.py:192; here it is one kernel);
* ``csr_segment_sum`` (fastmd/models/matris/op/triton_csr_segment_sum.py:433) and
  ``segment_csr`` (its CSR metadata, triton_segment_attention.py:824);
* ``segment_count`` / ``aggregate`` (fastmd/engine/kernels/segment.py:42 / :97).

Every op is a ``torch.autograd.Function`` whose forward and backward are
kernels of libfastmd_b200.so called through its C ABI on torch's current
stream (no host synchronisation: capturable in a CUDA graph). The backward
passes of the gathers reduce through a CSR of the gather index instead of
atomics, so every gradient is deterministic. CUDA tensors only: there is no
CPU path.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading

import torch
from torch import Tensor
from torch.autograd import Function

from fastmd_b200 import _lib
from fastmd_b200._lib import FmdCatPart, call, ptr, stream


def _rows_view(matrix: Tensor) -> tuple[Tensor, int]:
    """``(matrix, row_stride)`` with unit column stride; copies only when needed."""
    if matrix.dim() != 2:
        raise ValueError(f"expected a 2D matrix, got shape {tuple(matrix.shape)}")
    if matrix.dtype != torch.float32:
        raise ValueError(f"fastmd_b200 edge/node ops take float32 rows, got {matrix.dtype}")
    if matrix.stride(1) != 1 and matrix.shape[1] > 1:
        matrix = matrix.contiguous()
    ld = matrix.stride(0) if matrix.shape[0] > 1 else max(matrix.shape[1], 1)
    return matrix, max(ld, matrix.shape[1])


def _index(index: Tensor) -> Tensor:
    if index.dim() != 1:
        raise ValueError(f"an index must be 1D, got shape {tuple(index.shape)}")
    return index.to(torch.int64).contiguous()


# ----------------------------------------------------------------------------- CSR metadata


_CSR_SCOPES: list[dict] = []  # process-wide: autograd runs a CUDA backward on its own device thread
_CSR_LOCK = threading.Lock()


@contextlib.contextmanager
def csr_scope():
    """Within the scope, ``segment_csr`` of the same index tensor (and segment count) is built once: a model
    evaluation whose layers gather, scatter and segment-reduce over the same few index tensors (forward and
    backward) sorts each index once. The scope is process-wide (the backward of an evaluation runs on
    autograd's device thread while the caller waits), so evaluations must not overlap in time. Entries hold
    their index tensor, so a key cannot be reused by another tensor in the scope; the cache dies with the
    scope. The indices must not change inside the scope."""
    with _CSR_LOCK:
        _CSR_SCOPES.append({})
    try:
        yield
    finally:
        with _CSR_LOCK:
            _CSR_SCOPES.pop()


def segment_csr(segment: Tensor, num_segment: int) -> tuple[Tensor, Tensor]:
    """``(perm, off)``: the rows grouped by segment (ascending row order inside a
    run, a stable sort) and the int64 run offsets ``[num_segment + 1]``.
    Replaces ``segment_attention_csr_metadata`` (triton_segment_attention.py:824)."""
    _lib.require_cuda(segment)
    if _CSR_SCOPES:
        cache = _CSR_SCOPES[-1]
        key = (id(segment), segment.data_ptr(), segment.shape[0], int(num_segment))
        hit = cache.get(key)
        if hit is None:
            hit = cache[key] = (segment, *_segment_csr(segment, num_segment))
        return hit[1], hit[2]
    return _segment_csr(segment, num_segment)


def _segment_csr(segment: Tensor, num_segment: int) -> tuple[Tensor, Tensor]:
    segment = _index(segment)
    rows, num_segment = segment.shape[0], int(num_segment)
    perm = torch.empty(rows, dtype=torch.int64, device=segment.device)
    off = torch.empty(num_segment + 1, dtype=torch.int64, device=segment.device)
    nbytes = ctypes.c_size_t(0)
    call("fmd_csr_build_workspace_bytes", rows, num_segment, ctypes.byref(nbytes))
    workspace = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=segment.device)
    call("fmd_csr_build", ptr(segment), rows, num_segment, ptr(perm), ptr(off), ptr(workspace),
         int(nbytes.value), ptr(_lib.flags_word(segment.device)), stream(segment.device))
    return perm, off


def csr_offsets(segment: Tensor, num_segment: int) -> Tensor:
    """Run offsets of an ascending ``segment`` (the identity CSR, dispatch.py:325-331)."""
    _lib.require_cuda(segment)
    segment = _index(segment)
    off = torch.empty(int(num_segment) + 1, dtype=torch.int64, device=segment.device)
    call("fmd_csr_offsets_sorted", ptr(segment), segment.shape[0], int(num_segment), ptr(off),
         stream(segment.device))
    return off


# ----------------------------------------------------------------------------- gather-cat


def _launch_gather_cat(parts: list[tuple[Tensor, int, Tensor | None, int]], rows: int, out: Tensor) -> None:
    array = (FmdCatPart * len(parts))()
    for k, (src, ld, index, width) in enumerate(parts):
        array[k].src = ptr(src)
        array[k].index = ptr(index) if index is not None else None
        array[k].ld = ld
        array[k].n_src = src.shape[0]
        array[k].width = width
    call("fmd_gather_cat", array, len(parts), rows, ptr(out), out.stride(0) if rows > 1 else out.shape[1],
         ptr(_lib.flags_word(out.device)), stream(out.device))


def _gather_bwd(grad: Tensor, gout: Tensor, col0: int, width: int, index: Tensor | None,
                accumulate: bool) -> None:
    """grad (=|+=) the CSR reduction of gout[:, col0:col0+width] over ``index``
    (None: the aligned block, a row copy)."""
    if index is None:
        call("fmd_copy_rows", ptr(gout[:, col0:]), gout.stride(0), ptr(grad), grad.stride(0), gout.shape[0],
             width, stream(gout.device))
        return
    perm, off = segment_csr(index, grad.shape[0])
    call("fmd_gather_rows_bwd", ptr(gout), gout.stride(0), col0, width, ptr(perm), ptr(off), grad.shape[0],
         ptr(grad), grad.stride(0), int(accumulate), stream(gout.device))


class _GatherCat(Function):
    """out = [parts...]; part k is ``src_k[index_k]`` (or ``src_k`` row-aligned)."""

    @staticmethod
    def forward(ctx, n_parts, *flat):
        srcs = list(flat[0::2][:n_parts])
        indices = list(flat[1::2][:n_parts])
        _lib.require_cuda(*srcs, *indices)
        rows = None
        for src, index in zip(srcs, indices):
            if index is None:
                rows = src.shape[0] if rows is None else rows
                if src.shape[0] != rows:
                    raise ValueError("aligned parts must have the same row count")
        for index in indices:
            if index is not None:
                n = index.shape[0]
                if rows is not None and n != rows:
                    raise ValueError(f"index has {n} rows, the aligned parts {rows}")
                rows = n
        launch, views = [], []
        for src, index in zip(srcs, indices):
            view, ld = _rows_view(src)
            idx = _index(index) if index is not None else None
            launch.append((view, ld, idx, view.shape[1]))
            views.append(idx)
        width = sum(p[3] for p in launch)
        out = torch.empty(rows, width, device=srcs[0].device, dtype=torch.float32)
        if rows > 0 and width > 0:
            _launch_gather_cat(launch, rows, out)
        ctx.save_for_backward(*[i for i in views if i is not None])
        ctx.has_index = [i is not None for i in views]
        ctx.shapes = [tuple(s.shape) for s in srcs]
        ctx.src_ids = [id(s) for s in srcs]
        return out

    @staticmethod
    def backward(ctx, gout):
        gout = gout.contiguous()
        saved = list(ctx.saved_tensors)
        grads: list[Tensor | None] = [None] * len(ctx.shapes)
        first_of: dict[int, int] = {}
        col0 = 0
        for k, shape in enumerate(ctx.shapes):
            index = saved.pop(0) if ctx.has_index[k] else None
            width = shape[1]
            owner = first_of.setdefault(ctx.src_ids[k], k)
            if ctx.needs_input_grad[1 + 2 * k] or ctx.needs_input_grad[1 + 2 * owner]:
                if grads[owner] is None:
                    grads[owner] = torch.empty(shape, device=gout.device, dtype=gout.dtype)
                    if shape[0] > 0 and width > 0:
                        _gather_bwd(grads[owner], gout, col0, width, index, accumulate=False)
                elif shape[0] > 0 and width > 0:
                    _gather_bwd(grads[owner], gout, col0, width, index, accumulate=True)
            col0 += width
        out = [None]
        for k in range(len(ctx.shapes)):
            out.extend([grads[k], None])
        return tuple(out)


def gather_cat(parts: list[tuple[Tensor, Tensor | None]]) -> Tensor:
    """``cat([src[index] or src for (src, index) in parts], 1)`` in one kernel, any widths.
    A source appearing in several parts (e.g. cat3's gathered rows) receives the
    sum of their gradients, in part order."""
    flat = []
    for src, index in parts:
        flat.extend([src, index])
    return _GatherCat.apply(len(parts), *flat)


def aligned_gather_cat3(aligned: Tensor, gathered: Tensor, index_a: Tensor, index_b: Tensor) -> Tensor:
    """``cat([aligned, gathered[index_a], gathered[index_b]], 1)`` (triton_gather_cat.py:181)."""
    if aligned.shape[1] != gathered.shape[1]:
        raise ValueError("aligned_gather_cat3 needs equal widths (use gather_cat for mixed widths)")
    return gather_cat([(aligned, None), (gathered, index_a), (gathered, index_b)])


def aligned_gather_cat4(aligned: Tensor, gathered_a: Tensor, index_a: Tensor, gathered_b: Tensor,
                        index_b: Tensor, index_c: Tensor) -> Tensor:
    """``cat([aligned, gathered_a[index_a], gathered_b[index_b], gathered_b[index_c]], 1)``
    (triton_gather_cat.py:353)."""
    if not (aligned.shape[1] == gathered_a.shape[1] == gathered_b.shape[1]):
        raise ValueError("aligned_gather_cat4 needs equal widths (use gather_cat for mixed widths)")
    return gather_cat([(aligned, None), (gathered_a, index_a), (gathered_b, index_b), (gathered_b, index_c)])


# ----------------------------------------------------------------------------- segment sums


class _CsrSegmentSum(Function):
    @staticmethod
    def forward(ctx, value, weight, segment, num_segment, perm, off, identity_perm, skip_segment):
        n_rows, dim = value.shape
        value, ldv = _rows_view(value)
        ldw = 0
        if weight is not None:
            weight, ldw = _rows_view(weight)
        if n_rows == 0:  # no rows: every segment sums to zero (nothing to read, nothing to launch)
            out = torch.zeros((num_segment, dim), device=value.device, dtype=value.dtype)
        else:
            out = torch.empty((num_segment, dim), device=value.device, dtype=value.dtype)
        if n_rows > 0 and num_segment > 0 and dim > 0:
            call("fmd_csr_segment_sum", ptr(value), ldv, ptr(weight), ldw,
                 None if identity_perm else ptr(perm), ptr(off), num_segment, dim, skip_segment, ptr(out),
                 dim, stream(value.device))
        ctx.save_for_backward(value, weight, segment)
        ctx.lds = (ldv, ldw)
        ctx.num_segment, ctx.skip_segment = num_segment, skip_segment
        return out

    @staticmethod
    def backward(ctx, gout):
        value, weight, segment = ctx.saved_tensors
        need_gv = ctx.needs_input_grad[0]
        need_gw = ctx.needs_input_grad[1] and weight is not None
        if not (need_gv or need_gw):
            return (None,) * 8
        gout = gout.contiguous()
        n_rows, dim = value.shape
        gvalue = torch.empty((n_rows, dim), device=value.device, dtype=value.dtype) if need_gv else None
        gweight = torch.empty((n_rows, dim), device=value.device, dtype=value.dtype) if need_gw else None
        if n_rows > 0 and dim > 0:
            ldv, ldw = ctx.lds
            call("fmd_csr_segment_sum_bwd", ptr(gout), ptr(value), ldv, ptr(weight), ldw, ptr(segment), n_rows,
                 ctx.num_segment, dim, ctx.skip_segment, ptr(gvalue), ptr(gweight),
                 ptr(_lib.flags_word(value.device)), stream(value.device))
        return gvalue, gweight, None, None, None, None, None, None


def csr_segment_sum(value: Tensor, segment: Tensor, num_segment: int, perm: Tensor | None = None,
                    off: Tensor | None = None, identity_perm: bool = False, *, weight: Tensor | None = None,
                    skip_segment: int = -1) -> Tensor:
    """``out[s] = sum_{segment[i] == s} [weight[i] *] value[i]`` over a CSR, deterministic.

    Same contract as triton_csr_segment_sum.py:433: ``perm``/``off`` the CSR of
    ``segment`` (built here when missing), ``identity_perm`` for rows sorted by
    segment (``off`` required), ``skip_segment`` -1 or a segment whose output is
    0 and whose rows get zero gradient.
    """
    if value.dim() != 2:
        raise ValueError(f"value must be 2D, got shape {tuple(value.shape)}")
    if weight is not None and (weight.shape != value.shape or weight.dtype != value.dtype):
        raise ValueError(
            f"weight must match value, got {tuple(weight.shape)}/{weight.dtype} and "
            f"{tuple(value.shape)}/{value.dtype}")
    n_rows = value.shape[0]
    if segment.dim() != 1 or segment.numel() != n_rows:
        raise ValueError(f"segment must have one entry per row ({n_rows}), got {tuple(segment.shape)}")
    num_segment = int(num_segment)
    skip_segment = int(skip_segment)
    if skip_segment < -1 or skip_segment >= num_segment:
        raise ValueError("skip_segment must be -1 or an existing private segment")
    identity_perm = bool(identity_perm)
    if identity_perm and off is None:
        raise ValueError("identity CSR metadata requires offsets")
    _lib.require_cuda(value, weight, segment, perm, off)
    if any(t is not None and t.device != value.device for t in (weight, segment, perm, off)):
        raise ValueError("value, weight, segment and the CSR must be on the same device")
    segment = _index(segment)
    if not identity_perm and (perm is None or off is None):
        perm, off = segment_csr(segment, num_segment)
    off = off.to(torch.int64).contiguous()
    if perm is not None:
        perm = perm.to(torch.int64).contiguous()
    return _CsrSegmentSum.apply(value, weight, segment, num_segment, perm, off, identity_perm, skip_segment)


def segment_count(segment: Tensor, num_segment: int) -> Tensor:
    """Rows per segment, int64 [num_segment], sync-free (segment.py:42)."""
    _, off = segment_csr(segment, num_segment)
    return off[1:] - off[:-1]


def aggregate(data: Tensor, segment: Tensor, bin_count: Tensor | None = None, average: bool = True,
              num_segment: int | None = None) -> Tensor:
    """Sum (or mean) of the rows of each segment (segment.py:97); ``num_segment`` is required
    here (the reference's ``bincount`` fallback syncs with the host)."""
    if num_segment is None:
        if bin_count is None:
            raise ValueError("aggregate needs num_segment or bin_count (no host synchronisation)")
        num_segment = bin_count.shape[0]
    perm, off = segment_csr(segment, int(num_segment))
    out = csr_segment_sum(data, segment, int(num_segment), perm, off)
    if average:
        if bin_count is None:
            bin_count = off[1:] - off[:-1]
        bin_count = bin_count.where(bin_count != 0, bin_count.new_ones(1))
        out = (out.T / bin_count).T
    return out


def read_flags(device=None, reset: bool = True) -> int:
    """The FMD_FLAG_* bits the op kernels raised on ``device`` (host read: a synchronisation)."""
    word = _lib.flags_word(device if device is not None else torch.cuda.current_device())
    value = int(word.item())
    if reset:
        word.zero_()
    return value
