"""Decomposed indexed-concat first linear with the fused gather-add + SiLU epilogue.

The operator surface of fastmd/engine/kernels/decomposed_indexed_cat_silu_linear.py
(``decomposed_indexed_cat3_silu_linear`` :892, ``decomposed_indexed_cat4_silu_linear`` :1002):

    cat3: [A | B[ia] | B[ib]] @ W^T + b   =  A W0^T + (B W1^T)[ia] + (B W2^T)[ib] + b
    cat4: [A | X[ia] | B[ib] | B[ic]] @ W^T + b

The projections run on the source rows (``wide_gemm.linear``: tcgen05 3xTF32, or the IEEE path),
then ``fmd_gather_add_silu`` gathers the projected rows, adds the bias and returns the SiLU of the
core and gate halves ``(core_act, gate_act)`` [rows, H] each. The backward's per-row SiLU derivative
is ``fmd_silu_pair_bwd``; its scatter into the gathered projections is the deterministic CSR row sum
``fmd_gather_rows_bwd`` (the reference's deterministic mode, without its atomics). Weights and bias
are frozen (no gradient), as in the reference. On a guard failure (CPU tensors, non-contiguous
sources or weights, a bias that is not 1-D) the functions return None like the reference's.
"""
from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd import Function

from . import _lib, wide_gemm
from ._lib import FmdCatPart, call, ptr, stream
from .ops import segment_csr


class _GatherAddSilu(Function):
    """(p0, bias, n, p_1..p_n, index_1..index_n) -> (core_act, gate_act)."""

    @staticmethod
    def forward(ctx, p0, bias, n, *args):
        ps, indices = args[:n], [i.to(torch.int64).contiguous() for i in args[n:]]
        rows, width = p0.shape[0], p0.shape[1]
        h = width // 2
        dev = p0.device
        pre = torch.empty((rows, width), device=dev, dtype=torch.float32)
        core = torch.empty((rows, h), device=dev, dtype=torch.float32)
        gate = torch.empty((rows, h), device=dev, dtype=torch.float32)
        parts = (FmdCatPart * max(n, 1))()
        for k, (p, idx) in enumerate(zip(ps, indices)):
            parts[k].src, parts[k].index, parts[k].ld, parts[k].n_src, parts[k].width = (
                ptr(p), ptr(idx), p.stride(0), p.shape[0], width)
        call("fmd_gather_add_silu", ptr(p0), p0.stride(0), parts, n, ptr(bias), rows, h, ptr(pre), ptr(core),
             ptr(gate), ptr(_lib.flags_word(dev)), stream(dev))
        ctx.save_for_backward(pre, *indices)
        ctx.n_src = [p.shape[0] for p in ps]
        ctx.n = n
        return core, gate

    @staticmethod
    def backward(ctx, grad_core, grad_gate):
        pre, *indices = ctx.saved_tensors
        rows, width = pre.shape
        h = width // 2
        dev = pre.device
        s = stream(dev)
        grad_core = torch.zeros((rows, h), device=dev) if grad_core is None else grad_core.contiguous()
        grad_gate = torch.zeros((rows, h), device=dev) if grad_gate is None else grad_gate.contiguous()
        grad_p0 = torch.empty((rows, width), device=dev, dtype=torch.float32)
        call("fmd_silu_pair_bwd", ptr(grad_core), ptr(grad_gate), ptr(pre), rows, h, ptr(grad_p0), width, s)
        grads = []
        for idx, n_src in zip(indices, ctx.n_src):
            perm, off = segment_csr(idx, n_src)
            g = torch.empty((n_src, width), device=dev, dtype=torch.float32)
            if n_src:
                call("fmd_gather_rows_bwd", ptr(grad_p0), width, 0, width, ptr(perm), ptr(off), n_src, ptr(g), width,
                     0, s)
            grads.append(g)
        return (grad_p0, None, None, *grads, *([None] * ctx.n))


def _ok(t: Tensor | None, *, contiguous: bool = True) -> bool:
    return t is not None and t.is_cuda and (t.is_contiguous() or not contiguous) and t.dtype == torch.float32


def _guards(aligned, sources, weights, n_weights, bias, precomputed_p0) -> bool:
    if precomputed_p0 is not None:
        if not (_ok(precomputed_p0, contiguous=False) and precomputed_p0.dim() == 2 and precomputed_p0.stride(1) == 1
                and precomputed_p0.shape[0] == aligned.shape[0] and precomputed_p0.shape[1] == weights[0].shape[0]):
            return False
    elif not _ok(aligned):
        return False
    if len(weights) != n_weights or not all(_ok(w) for w in weights) or not all(_ok(x) for x in sources):
        return False
    if bias is not None and not (_ok(bias) and bias.dim() == 1 and bias.numel() == weights[0].shape[0]):
        return False
    if any(w.requires_grad for w in weights) or (bias is not None and bias.requires_grad):
        return False  # frozen projections only (the wide GEMM has no weight gradient)
    return weights[0].shape[0] % 2 == 0


def decomposed_indexed_cat3_silu_linear(aligned: Tensor, gathered: Tensor, index_a: Tensor, index_b: Tensor,
                                        weights: tuple[Tensor, Tensor, Tensor], bias: Tensor | None = None,
                                        index_a_sorted: bool = False, precomputed_p0: Tensor | None = None, *,
                                        strict_errors: bool = False,
                                        precision: str = "tf32x3") -> tuple[Tensor, Tensor] | None:
    """``silu`` halves of ``[aligned | gathered[index_a] | gathered[index_b]] @ W^T + bias`` with
    ``W = [W0 | W1 | W2]`` (``weights``, each [2H, D]); ``(core_act, gate_act)`` or None when a guard
    declines. ``index_a_sorted`` is accepted for the reference's signature (the CSR scatter of the
    backward needs no sorted pairing)."""
    del index_a_sorted, strict_errors
    if not _guards(aligned, (gathered,), weights, 3, bias, precomputed_p0):
        return None
    p0 = precomputed_p0 if precomputed_p0 is not None else wide_gemm.linear(aligned, weights[0], precision=precision)
    p1 = wide_gemm.linear(gathered, weights[1], precision=precision)
    p2 = wide_gemm.linear(gathered, weights[2], precision=precision)
    return _GatherAddSilu.apply(p0, bias, 2, p1, p2, index_a, index_b)


def decomposed_indexed_cat4_silu_linear(aligned: Tensor, gathered_a: Tensor, index_a: Tensor, gathered_b: Tensor,
                                        index_b: Tensor, index_c: Tensor,
                                        weights: tuple[Tensor, Tensor, Tensor, Tensor], bias: Tensor | None = None,
                                        index_a_sorted: bool = False, precomputed_p0: Tensor | None = None, *,
                                        strict_errors: bool = False,
                                        precision: str = "tf32x3") -> tuple[Tensor, Tensor] | None:
    """As ``decomposed_indexed_cat3_silu_linear`` for ``[aligned | gathered_a[index_a] | gathered_b[index_b] |
    gathered_b[index_c]]``."""
    del index_a_sorted, strict_errors
    if not _guards(aligned, (gathered_a, gathered_b), weights, 4, bias, precomputed_p0):
        return None
    p0 = precomputed_p0 if precomputed_p0 is not None else wide_gemm.linear(aligned, weights[0], precision=precision)
    p1 = wide_gemm.linear(gathered_a, weights[1], precision=precision)
    p2 = wide_gemm.linear(gathered_b, weights[2], precision=precision)
    p3 = wide_gemm.linear(gathered_b, weights[3], precision=precision)
    return _GatherAddSilu.apply(p0, bias, 3, p1, p2, p3, index_a, index_b, index_c)
