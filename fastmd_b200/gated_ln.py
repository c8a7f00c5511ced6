"""The MatRIS GatedMLP epilogue: ``silu(LN(core)) * sigmoid(LN(gate))`` (+ a weighted residual).

The operator surface of fastmd/models/matris/op/triton_gated_ln.py: ``fused_gated_ln`` (:718) and
``fused_gated_ln_residual`` (:750), frozen LayerNorm parameters, gradients for the core/gate inputs, the
residual, and the folded linear biases ``core_lb``/``gate_lb`` when they require them (their column
sums). Kernels: ``fmd_gated_ln`` / ``fmd_gated_ln_bwd`` / ``fmd_column_sum``
(fastmd_b200/csrc/gated_ln.cu). Where the reference falls back to its unfused path (CPU tensors,
trainable LayerNorm parameters), this build raises: there is no CPU path, and the LayerNorm weights of
the frozen models are not trained here. Mismatched shapes raise ``ValueError``.
"""
from __future__ import annotations

import ctypes

import torch
from torch import Tensor
from torch.autograd import Function

from . import _lib
from ._lib import FastMDLibraryError, call, ptr, stream


def _column_sum(x: Tensor) -> Tensor:
    rows, cols = x.shape
    nbytes = ctypes.c_size_t(0)
    call("fmd_column_sum_workspace_bytes", rows, cols, ctypes.byref(nbytes))
    ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=x.device)
    out = torch.empty(cols, dtype=torch.float32, device=x.device)
    call("fmd_column_sum", ptr(x), rows, cols, x.stride(0), ptr(ws), ws.numel(), ptr(out), stream(x.device))
    return out


class _GatedLN(Function):
    @staticmethod
    def forward(ctx, core_x, gate_x, core_w, core_b, gate_w, gate_b, residual, res_weight, eps_core, eps_gate,
                core_lb, gate_lb):
        core_x, gate_x = core_x.contiguous(), gate_x.contiguous()
        params = [p.contiguous() for p in (core_w, core_b, gate_w, gate_b)]
        core_lb = core_lb.contiguous() if core_lb is not None else None
        gate_lb = gate_lb.contiguous() if gate_lb is not None else None
        residual = residual.contiguous() if residual is not None else None
        res_weight = res_weight.contiguous() if res_weight is not None else None
        rows, dim = core_x.shape
        dev = core_x.device
        out = torch.empty_like(core_x)
        stats = [torch.empty(rows, dtype=torch.float32, device=dev) for _ in range(4)]
        call("fmd_gated_ln", ptr(core_x), ptr(gate_x), ptr(core_lb), ptr(gate_lb), *map(ptr, params), ptr(residual),
             ptr(res_weight), rows, dim, float(eps_core), float(eps_gate), ptr(out), *map(ptr, stats), stream(dev))
        ctx.save_for_backward(core_x, gate_x, *params, core_lb, gate_lb, res_weight, *stats)
        ctx.has_residual = residual is not None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        core_x, gate_x, cw, cb, gw, gb, core_lb, gate_lb, res_weight, *stats = ctx.saved_tensors
        rows, dim = core_x.shape
        dev = core_x.device
        grad_out = grad_out.contiguous()
        gcx, ggx = torch.empty_like(core_x), torch.empty_like(gate_x)
        gres = torch.empty_like(core_x) if ctx.has_residual else None
        call("fmd_gated_ln_bwd", ptr(core_x), ptr(gate_x), ptr(core_lb), ptr(gate_lb), ptr(cw), ptr(cb), ptr(gw),
             ptr(gb), ptr(res_weight), ptr(grad_out), *map(ptr, stats), rows, dim, ptr(gcx), ptr(ggx), ptr(gres),
             stream(dev))
        glb_c = _column_sum(gcx) if ctx.needs_input_grad[10] else None
        glb_g = _column_sum(ggx) if ctx.needs_input_grad[11] else None
        return gcx, ggx, None, None, None, None, gres, None, None, None, glb_c, glb_g


def _check(core_x, gate_x, params, residual=None, res_weight=None):
    _lib.require_cuda(core_x, gate_x, *params, residual, res_weight)
    if core_x.shape != gate_x.shape or core_x.dim() != 2 or (residual is not None and residual.shape != core_x.shape):
        raise ValueError("core_x, gate_x (and residual) must be [rows, width] of one shape")
    if res_weight is not None and core_x.shape[1] != res_weight.numel():
        raise ValueError("res_weight must have the row width")
    if any(p is not None and p.requires_grad for p in params + [res_weight]):
        raise FastMDLibraryError("gated LN: trainable LayerNorm / residual weights are not supported (frozen models)")
    if core_x.shape[1] > 256:
        raise FastMDLibraryError("gated LN: row width above 256")


def fused_gated_ln(core_x: Tensor, gate_x: Tensor, core_w: Tensor, core_b: Tensor, gate_w: Tensor, gate_b: Tensor,
                   eps_core: float = 1e-5, eps_gate: float = 1e-5, core_lb: Tensor | None = None,
                   gate_lb: Tensor | None = None) -> Tensor:
    """``silu(LN(core_x + core_lb)) * sigmoid(LN(gate_x + gate_lb))`` (triton_gated_ln.py:718)."""
    if (core_lb is None) != (gate_lb is None):
        raise ValueError("core_lb and gate_lb: both or neither")
    _check(core_x, gate_x, [core_w, core_b, gate_w, gate_b])
    return _GatedLN.apply(core_x, gate_x, core_w, core_b, gate_w, gate_b, None, None, eps_core, eps_gate, core_lb,
                          gate_lb)


def fused_gated_ln_residual(core_x: Tensor, gate_x: Tensor, core_w: Tensor, core_b: Tensor, gate_w: Tensor,
                            gate_b: Tensor, residual: Tensor, res_weight: Tensor, eps_core: float = 1e-5,
                            eps_gate: float = 1e-5, core_lb: Tensor | None = None,
                            gate_lb: Tensor | None = None) -> Tensor:
    """``fused_gated_ln(...) + res_weight * residual`` (triton_gated_ln.py:750)."""
    if (core_lb is None) != (gate_lb is None):
        raise ValueError("core_lb and gate_lb: both or neither")
    _check(core_x, gate_x, [core_w, core_b, gate_w, gate_b], residual, res_weight)
    return _GatedLN.apply(core_x, gate_x, core_w, core_b, gate_w, gate_b, residual, res_weight, eps_core, eps_gate,
                          core_lb, gate_lb)
