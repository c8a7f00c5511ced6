"""Segment attention: the MatRIS receiver softmax-weighted sum, on a CSR.

The operator surface of fastmd/models/matris/op/triton_segment_attention.py: ``segment_attention``
(:870), ``paired_segment_attention`` (:918) and ``segment_attention_csr_metadata`` (:824), with the
reference's argument meaning, outputs and errors (``ValueError`` for mismatched shapes, non-2-D logits,
an invalid ``skip_segment`` or identity CSR metadata without offsets). The kernels are
``fmd_segment_attention`` / ``fmd_segment_attention_bwd`` / ``fmd_paired_segment_attention_bwd_rows``
(fastmd_b200/csrc/segment_attention.cu). Tensors must live on a CUDA device: there is no CPU path.
"""
from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd import Function

from . import _lib
from ._lib import call, ptr, stream
from .ops import csr_offsets, segment_csr


def segment_attention_csr_metadata(segment: Tensor, num_segment: int) -> tuple[Tensor, Tensor]:
    """``(perm, off)``: rows grouped by segment (stable) and int64 offsets ``[num_segment + 1]``."""
    return segment_csr(segment, int(num_segment))


def _rows2d(x: Tensor) -> Tensor:
    return x if x.stride(1) == 1 else x.contiguous()


def _check_skip(skip_segment: int, num_segment: int) -> None:
    if skip_segment < -1 or skip_segment >= num_segment:
        raise ValueError("skip_segment must be -1 or an existing private segment")


def _csr(segment: Tensor, num_segment: int, perm, off, identity: bool, side: str = "") -> tuple[Tensor | None, Tensor]:
    if identity and off is None:
        raise ValueError(f"identity CSR metadata{side} requires offsets")
    if identity:
        return None, off.to(torch.int64)
    if perm is None or off is None:
        perm, off = segment_csr(segment, num_segment)
    return perm.to(torch.int64), off.to(torch.int64)


def _forward(logits, value, perm, off, num_segment, skip, *, lse=False, stats=False):
    rows, dim = logits.shape
    dev = logits.device
    out = torch.empty((num_segment, dim), device=dev, dtype=torch.float32)
    ls = torch.empty_like(out) if lse else None
    mx = torch.empty_like(out) if stats else None
    dn = torch.empty_like(out) if stats else None
    call("fmd_segment_attention", ptr(logits), logits.stride(0), ptr(value), value.stride(0), ptr(perm), ptr(off),
         rows, num_segment, dim, skip, ptr(out), ptr(ls), ptr(mx), ptr(dn), ptr(_lib.flags_word(dev)), stream(dev))
    return out, ls, mx, dn


class _SegmentAttention(Function):
    @staticmethod
    def forward(ctx, logits, value, segment, num_segment, perm, off, identity_perm, skip_segment, return_lse):
        logits, value = _rows2d(logits), _rows2d(value)
        perm, off = _csr(segment, num_segment, perm, off, identity_perm)
        out, lse, _, _ = _forward(logits, value, perm, off, num_segment, skip_segment, lse=return_lse)
        ctx.save_for_backward(logits, value, perm, off, out)
        ctx.skip_segment = skip_segment
        # a provided CSR may cover a subset of the rows; its backward visits only those
        ctx.partial_rows = perm is not None and perm.numel() != logits.shape[0]
        return (out, lse) if return_lse else out

    @staticmethod
    def backward(ctx, gout, glse=None):
        logits, value, perm, off, out = ctx.saved_tensors
        rows, dim = logits.shape
        dev = logits.device
        gout = gout.contiguous()
        glse = glse.contiguous() if glse is not None else None
        zero_init = ctx.skip_segment >= 0 or ctx.partial_rows
        alloc = torch.zeros if zero_init else torch.empty
        grad_logits = alloc((rows, dim), device=dev, dtype=torch.float32)
        grad_value = alloc((rows, dim), device=dev, dtype=torch.float32)
        call("fmd_segment_attention_bwd", ptr(logits), logits.stride(0), ptr(value), value.stride(0), ptr(out),
             ptr(gout), ptr(glse), ptr(perm), ptr(off), rows, out.shape[0], dim, ctx.skip_segment, ptr(grad_logits),
             dim, ptr(grad_value), dim, ptr(_lib.flags_word(dev)), stream(dev))
        return grad_logits, grad_value, None, None, None, None, None, None, None


def segment_attention(logits: Tensor, value: Tensor, segment: Tensor, num_segment: int, perm: Tensor | None = None,
                      off: Tensor | None = None, identity_perm: bool = False, *, skip_segment: int = -1,
                      return_lse: bool = False) -> Tensor | tuple[Tensor, Tensor]:
    """``out[s] = sum_i softmax(logits over segment s)_i * value_i`` per column; ``return_lse`` also
    returns ``lse = max + log(denom)`` (-inf for an empty or skipped segment, whose ``out`` is 0).
    ``identity_perm``: the rows are sorted by segment and ``off`` is given."""
    _lib.require_cuda(logits, value, segment, perm, off)
    if logits.shape != value.shape:
        raise ValueError(f"logits and value must have the same shape, got {logits.shape} and {value.shape}")
    if logits.dim() != 2:
        raise ValueError(f"logits must be 2D, got shape {logits.shape}")
    num_segment, skip_segment = int(num_segment), int(skip_segment)
    _check_skip(skip_segment, num_segment)
    return _SegmentAttention.apply(logits, value, segment, num_segment, perm, off, bool(identity_perm), skip_segment,
                                   bool(return_lse))


class _PairedSegmentAttention(Function):
    @staticmethod
    def forward(ctx, logits_a, logits_b, value, segment_a, segment_b, num_segment, perm_a, off_a, perm_b, off_b,
                identity_a, identity_b, skip_segment, return_lse):
        logits_a, logits_b, value = _rows2d(logits_a), _rows2d(logits_b), _rows2d(value)
        segment_a = segment_a.to(torch.int64).contiguous()
        segment_b = segment_b.to(torch.int64).contiguous()
        perm_a, off_a = _csr(segment_a, num_segment, perm_a, off_a, identity_a, " for segment_a")
        perm_b, off_b = _csr(segment_b, num_segment, perm_b, off_b, identity_b, " for segment_b")
        out_a, lse_a, max_a, den_a = _forward(logits_a, value, perm_a, off_a, num_segment, skip_segment,
                                              lse=return_lse, stats=True)
        out_b, lse_b, max_b, den_b = _forward(logits_b, value, perm_b, off_b, num_segment, skip_segment,
                                              lse=return_lse, stats=True)
        ctx.save_for_backward(logits_a, logits_b, value, segment_a, segment_b, out_a, out_b, max_a, den_a, max_b,
                              den_b)
        ctx.skip_segment = skip_segment
        return (out_a, out_b, lse_a, lse_b) if return_lse else (out_a, out_b)

    @staticmethod
    def backward(ctx, gout_a, gout_b, glse_a=None, glse_b=None):
        logits_a, logits_b, value, segment_a, segment_b, out_a, out_b, max_a, den_a, max_b, den_b = ctx.saved_tensors
        rows, dim = logits_a.shape
        dev = logits_a.device
        gout_a, gout_b = gout_a.contiguous(), gout_b.contiguous()
        if (glse_a is None) != (glse_b is None):  # one side's lse unused: its cotangent is zero
            glse_a = torch.zeros_like(out_a) if glse_a is None else glse_a
            glse_b = torch.zeros_like(out_b) if glse_b is None else glse_b
        glse_a = glse_a.contiguous() if glse_a is not None else None
        glse_b = glse_b.contiguous() if glse_b is not None else None
        grad_a = torch.empty((rows, dim), device=dev, dtype=torch.float32)
        grad_b = torch.empty((rows, dim), device=dev, dtype=torch.float32)
        grad_value = torch.empty((rows, dim), device=dev, dtype=torch.float32)
        call("fmd_paired_segment_attention_bwd_rows", ptr(logits_a), logits_a.stride(0), ptr(logits_b),
             logits_b.stride(0), ptr(value), value.stride(0), ptr(gout_a), ptr(gout_b), ptr(out_a), ptr(out_b),
             ptr(max_a), ptr(den_a), ptr(max_b), ptr(den_b), ptr(segment_a), ptr(segment_b), ptr(glse_a), ptr(glse_b),
             rows, out_a.shape[0], dim, ctx.skip_segment, ptr(grad_a), dim, ptr(grad_b), dim, ptr(grad_value),
             ptr(_lib.flags_word(dev)), stream(dev))
        return grad_a, grad_b, grad_value, *([None] * 11)


def paired_segment_attention(logits_a: Tensor, logits_b: Tensor, value: Tensor, segment_a: Tensor, segment_b: Tensor,
                             num_segment: int, perm_a: Tensor | None = None, off_a: Tensor | None = None,
                             perm_b: Tensor | None = None, off_b: Tensor | None = None, identity_a: bool = False,
                             identity_b: bool = False, *, skip_segment: int = -1,
                             return_lse: bool = False) -> tuple[Tensor, ...]:
    """Two segment attentions of the same rows sharing ``value``: ``(out_a, out_b)``, and
    ``(lse_a, lse_b)`` after them with ``return_lse``; ``skip_segment`` as in ``segment_attention``."""
    _lib.require_cuda(logits_a, logits_b, value, segment_a, segment_b, perm_a, off_a, perm_b, off_b)
    if logits_a.shape != logits_b.shape or logits_a.shape != value.shape:
        raise ValueError("logits_a, logits_b, and value must have the same shape, got "
                         f"{logits_a.shape}, {logits_b.shape}, {value.shape}")
    if logits_a.dim() != 2:
        raise ValueError(f"logits must be 2D, got {logits_a.shape}")
    num_segment, skip_segment = int(num_segment), int(skip_segment)
    _check_skip(skip_segment, num_segment)
    return _PairedSegmentAttention.apply(logits_a, logits_b, value, segment_a, segment_b, num_segment, perm_a, off_a,
                                         perm_b, off_b, bool(identity_a), bool(identity_b), skip_segment,
                                         bool(return_lse))


__all__ = ["segment_attention", "paired_segment_attention", "segment_attention_csr_metadata", "csr_offsets"]
