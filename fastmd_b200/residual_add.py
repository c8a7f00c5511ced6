"""The MatRIS residual add with a frozen per-column weight.

The operator surface of fastmd/models/matris/op/triton_residual_add.py: ``residual_add(delta, residual,
weight)`` (:163) returns ``delta + residual * weight[None, :]``; its backward gives ``grad_delta = gout``
and ``grad_residual = gout * weight`` and no weight gradient (the weight is frozen: the reference's
dispatcher takes this op only when ``not weight.requires_grad``, dispatch.py:265). Both directions run
in ``fmd_residual_add`` (fastmd_b200/csrc/residual_add.cu), bit-identical to the reference's kernels
(the product rounded before the addition). Row-strided views with unit column stride (``packed[:, :D]``)
are read in place; any other layout is copied, as the reference does (:91-104); the output is a fresh
contiguous tensor. There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd import Function

from ._lib import call, ptr, require_cuda, stream

FORWARD, BACKWARD = 0, 1


def _rows(t: Tensor) -> Tensor:
    """``t`` with unit column stride (its row stride kept)."""
    return t if t.stride(1) == 1 and t.stride(0) >= max(t.shape[1], 1) else t.contiguous()


def _launch(op: int, delta: Tensor | None, residual: Tensor, weight: Tensor) -> Tensor:
    n, d = residual.shape
    out = torch.empty((n, d), device=residual.device, dtype=torch.float32)
    call("fmd_residual_add", op, ptr(delta), 0 if delta is None else delta.stride(0), ptr(residual),
         residual.stride(0), ptr(weight), n, d, ptr(out), d, stream(residual.device))
    return out


class _ResidualAdd(Function):
    @staticmethod
    def forward(ctx, delta, residual, weight):
        weight = weight.reshape(-1).contiguous()
        ctx.save_for_backward(weight)
        return _launch(FORWARD, _rows(delta), _rows(residual), weight)

    @staticmethod
    def backward(ctx, gout):
        (weight,) = ctx.saved_tensors
        return gout, _launch(BACKWARD, None, _rows(gout), weight), None


def residual_add(delta: Tensor, residual: Tensor, weight: Tensor) -> Tensor:
    """``delta + residual * weight[None, :]`` over ``[N, D]`` float32 CUDA tensors (``weight`` holds D
    values, any shape); differentiable in ``delta`` and ``residual``."""
    if delta.dim() != 2 or residual.shape != delta.shape or weight.numel() != delta.shape[1]:
        raise ValueError(f"residual_add: delta {tuple(delta.shape)} and residual {tuple(residual.shape)} must be "
                         f"the same [N, D] and weight ({weight.numel()} values) must hold D")
    if not (delta.dtype == residual.dtype == weight.dtype == torch.float32):
        raise TypeError("residual_add: this build computes in float32")
    require_cuda(delta, residual, weight)
    if delta.shape[1] == 0:
        return torch.empty_like(delta, memory_format=torch.contiguous_format)
    return _ResidualAdd.apply(delta, residual, weight)


__all__ = ["residual_add"]
