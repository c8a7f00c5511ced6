"""Wide frozen-weight GEMMs on the tcgen05 tensor cores at FP32 accuracy (3xTF32).

The operator surface of fastmd/engine/kernels/triton_wide_gemm.py: ``linear`` (:482), ``linear_into``
(:518), ``matmul`` (:534), ``wide_gemm_decline`` (:227) and the per-weight-version split cache
(``_split`` :188). ``y = x W^T (+ b) (+ c)`` and ``dX = dY W (+ c)`` run in ``fmd_gemm_tf32x3``
(fastmd_b200/csrc/gemm_tcgen05.cu): TMA tiles of x and of the weight's TF32 hi/lo pair, tcgen05.mma
kind::tf32 into TMEM, ``x_lo w_hi + x_hi w_lo + x_hi w_hi`` per 64-wide K chunk on a fresh accumulator,
the chunks summed in FP32, then bias, residual and (optionally) SiLU in the epilogue.

``precision``: ``"tf32x3"`` (the tensor-core path) or ``"ieee"`` (``fmd_gemm_f32``, one FP32 FMA chain
per output on the CUDA cores: the TF32-off parity path where the reference runs cuBLAS FP32). The weight
is frozen (no weight gradient), as in the reference. Tensors must live on a CUDA device: there is no CPU
path.

Differences from the reference's dispatch, by design: the kernel takes any ``K, N >= 1`` (the reference
declines ``K % 16``, ``N`` not 128-tiled, and ``K, N < 64`` to cuBLAS), so ``wide_gemm_decline`` reports
only shape, device, dtype, trainable-parameter and layout reasons; there is no row threshold (every
call takes the kernel it asks for).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch.autograd import Function
from torch.utils.weak import WeakIdKeyDictionary

from ._lib import FastMDLibraryError, call, ptr, require_cuda, stream

PRECISIONS = ("tf32x3", "ieee")


@dataclass
class _Split:
    """The TF32 pair of one weight orientation: ``hi`` / ``lo`` K-major [n, k], row stride a multiple of 4."""

    hi: torch.Tensor
    lo: torch.Tensor
    version: int
    pointer: int


# weight -> {(shape, strides, offset, transposed): _Split}; entries die with the weight
_SPLITS: WeakIdKeyDictionary = WeakIdKeyDictionary()


def _split(weight: torch.Tensor, transposed: bool, build: bool = True) -> _Split | None:
    """The hi/lo pair of ``weight`` (``[n, k]``), or of ``weight^T`` when ``transposed`` (the operand of
    ``dY @ W``), rebuilt when the weight's version or storage changed (triton_wide_gemm.py:188)."""
    entries = _SPLITS.get(weight)
    if entries is None:
        if not build:
            return None
        entries = _SPLITS[weight] = {}
    key = (tuple(weight.shape), tuple(weight.stride()), weight.storage_offset(), transposed)
    split = entries.get(key)
    if split is not None and split.version == weight._version and split.pointer == weight.data_ptr():
        return split
    if not build:
        return None
    w = weight.detach()
    if w.stride(1) != 1:
        w = w.contiguous()
    rows, cols = w.shape
    n, k = (cols, rows) if transposed else (rows, cols)
    ld = (k + 3) // 4 * 4  # TMA: row strides in multiples of 16 bytes
    hi = torch.empty((n, ld), dtype=torch.float32, device=w.device)[:, :k]
    lo = torch.empty((n, ld), dtype=torch.float32, device=w.device)[:, :k]
    call("fmd_tf32_split", ptr(w), rows, cols, w.stride(0), int(transposed), ptr(hi), ptr(lo), ld, stream(w.device))
    split = entries[key] = _Split(hi, lo, weight._version, weight.data_ptr())
    return split


def wide_gemm_decline(a: torch.Tensor, w: torch.Tensor, transposed: bool, bias=None, c=None, out=None) -> str | None:
    """None if ``a @ B`` (``B = w^T``, or ``w`` when ``transposed``) runs in ``fmd_gemm_tf32x3``, else why not
    (the reasons of triton_wide_gemm.py:227)."""
    k = a.shape[-1] if a.dim() == 2 else -1
    n = w.shape[1] if transposed else w.shape[0]
    if a.dim() != 2 or w.dim() != 2 or (w.shape[0] if transposed else w.shape[1]) != k or k < 1 or n < 1:
        return "shape"
    if not (a.is_cuda and w.device == a.device):
        return "device"
    if a.dtype != torch.float32 or w.dtype != torch.float32 or torch.is_autocast_enabled("cuda"):
        return "dtype"
    if w.requires_grad or (bias is not None and bias.requires_grad):
        return "trainable_params"
    if (a.stride(1) != 1 or a.stride(0) % 4 or a.stride(0) < k or a.data_ptr() % 16
            or (c is not None and (c.stride(1) != 1 or c.shape != (a.shape[0], n)))
            or (out is not None and (out.stride(1) != 1 or out.shape != (a.shape[0], n)))):
        return "layout"
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous() or bias.numel() != n):
        return "layout"
    return None


def _launch(a: torch.Tensor, weight: torch.Tensor, transposed: bool, precision: str, bias=None, c=None, out=None,
            act: int = 0) -> torch.Tensor:
    """y = act(a @ B + bias + c), B = weight^T (or weight when ``transposed``), into ``out`` or a new tensor."""
    m, k = a.shape
    n = weight.shape[1] if transposed else weight.shape[0]
    y = torch.empty((m, n), device=a.device, dtype=torch.float32) if out is None else out
    if m == 0:
        return y
    s = stream(a.device)
    if precision == "tf32x3":
        split = _split(weight, transposed)
        call("fmd_gemm_tf32x3", ptr(a), a.stride(0), ptr(split.hi), ptr(split.lo), split.hi.stride(0), ptr(bias),
             ptr(c), c.stride(0) if c is not None else 0, ptr(y), y.stride(0), m, n, k, act, 0, None, s)
        return y
    # IEEE FP32 on the CUDA cores: y = c, then y += act(a . B + bias)
    w = weight.detach()
    if w.stride(1) != 1:
        w = w.contiguous()
    if c is not None and c.data_ptr() != y.data_ptr():
        y.copy_(c)
    call("fmd_gemm_f32", ptr(a), a.stride(0), None, 0, ptr(w), w.stride(0), int(not transposed), ptr(bias), ptr(y),
         y.stride(0), None, 0, m, n, k, act, int(c is not None), s)
    return y


def grouped(problems) -> list[torch.Tensor]:
    """Up to 4 independent ``_launch(a, weight, transposed, "tf32x3", bias, c, out, act)`` problems in one
    ``fmd_gemm_tf32x3_grouped`` launch (each result bitwise that of its own call); ``problems`` are dicts
    with keys a, weight and optionally transposed, bias, c, out, act. Returns the outputs."""
    from ._lib import FmdGemmProblem

    if not 1 <= len(problems) <= 4:
        raise ValueError("one to four problems per grouped launch")
    arr = (FmdGemmProblem * len(problems))()
    outs, keep = [], []
    for i, q in enumerate(problems):
        a, weight = q["a"], q["weight"]
        transposed = q.get("transposed", False)
        m, k = a.shape
        n = weight.shape[1] if transposed else weight.shape[0]
        out = q.get("out")
        y = torch.empty((m, n), device=a.device, dtype=torch.float32) if out is None else out
        split = _split(weight, transposed)
        c, bias = q.get("c"), q.get("bias")
        arr[i] = FmdGemmProblem(ptr(a), a.stride(0), ptr(split.hi), ptr(split.lo), split.hi.stride(0), ptr(bias),
                                ptr(c), c.stride(0) if c is not None else 0, ptr(y), y.stride(0), m, n, k,
                                int(q.get("act", 0)), 0)
        outs.append(y)
        keep.append(split)
    call("fmd_gemm_tf32x3_grouped", arr, len(problems), None, stream(problems[0]["a"].device))
    return outs


def _check(a, weight, transposed, bias=None, c=None, out=None, precision="tf32x3") -> torch.Tensor:
    """``a`` in a layout the kernel takes (a copy fixes a row stride or base the TMA cannot use: a row's
    result does not depend on it), after the checks of ``wide_gemm_decline``."""
    require_cuda(a, weight, bias, c, out)
    if precision not in PRECISIONS:
        raise ValueError(f"precision must be one of {PRECISIONS}, got {precision!r}")
    if a.dim() == 2 and (a.stride(1) != 1 or a.stride(0) % 4 or a.data_ptr() % 16):
        k = a.shape[1]
        buf = torch.zeros((a.shape[0], (k + 3) // 4 * 4), dtype=a.dtype, device=a.device)
        buf[:, :k] = a
        a = buf[:, :k]
    why = wide_gemm_decline(a, weight, transposed, bias, c, out)
    if why is not None:
        raise FastMDLibraryError(f"wide GEMM declined: {why}")
    return a


class _WideLinear(Function):
    """``linear`` with an input gradient ``dY @ W`` through the same kernel (frozen weight)."""

    @staticmethod
    def forward(ctx, x, weight, bias, precision):
        ctx.save_for_backward(weight)
        ctx.precision = precision
        return _launch(x, weight, False, precision, bias)

    @staticmethod
    def backward(ctx, grad):
        (weight,) = ctx.saved_tensors
        g = _check(grad.contiguous(), weight, True, precision=ctx.precision)
        return _launch(g, weight, True, ctx.precision), None, None, None


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, precision: str = "tf32x3",
           act: int = 0) -> torch.Tensor:
    """``F.linear(x, weight, bias)`` of a frozen layer (then SiLU when ``act == 1``, forward only), with
    the input gradient on the same kernel (triton_wide_gemm.py:482)."""
    x = _check(x, weight, False, bias, precision=precision)
    if torch.is_grad_enabled() and x.requires_grad:
        if act:
            raise ValueError("act=1 is forward-only; apply SiLU outside the GEMM for autograd")
        return _WideLinear.apply(x, weight, bias, precision)
    return _launch(x, weight, False, precision, bias, act=act)


def linear_into(out: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                rows: int | None = None, precision: str = "tf32x3", act: int = 0) -> torch.Tensor:
    """``out[:] = x @ weight^T (+ bias)`` with no autograd (triton_wide_gemm.py:518). ``rows`` is accepted
    for the reference's signature; a row's result never depends on the row count here."""
    del rows
    x = _check(x, weight, False, bias, out=out, precision=precision)
    return _launch(x, weight, False, precision, bias, out=out, act=act)


def matmul(grad: torch.Tensor, weight: torch.Tensor, c: torch.Tensor | None = None, rows: int | None = None,
           accumulate: bool = False, enabled: bool | None = None, precision: str = "tf32x3") -> torch.Tensor:
    """``grad @ weight (+ c)`` for a frozen ``weight`` (an input gradient ``dY @ W``, no autograd;
    triton_wide_gemm.py:534). ``accumulate``: written into ``c`` in place (each element of ``c`` is read
    before the same thread stores it), else a new tensor. ``rows`` and ``enabled`` are accepted for the
    reference's signature (there is no dispatch threshold here)."""
    del rows, enabled
    grad = _check(grad, weight, True, c=c, precision=precision)
    if accumulate and c is None:
        raise ValueError("accumulate=True needs c")
    return _launch(grad, weight, True, precision, c=c, out=c if accumulate else None)
