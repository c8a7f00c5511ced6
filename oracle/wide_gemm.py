"""CPU restatement of the reference's 3xTF32 wide GEMM -- TEST INFRASTRUCTURE ONLY.

Restates fastmd/engine/kernels/triton_wide_gemm.py:
  * ``_rna_tf32`` (:63): ``cvt.rna.tf32.f32``, round to nearest with ties away from zero to TF32
    (10 explicit mantissa bits, the low 13 bits of the FP32 pattern zero);
  * ``_split_kernel`` (:132): ``hi = rna_tf32(w)``, ``lo = w - hi``;
  * ``_k_chunk`` / ``_tile`` (:69, :83): per 64-wide K chunk a fresh accumulator of
    ``a_lo b_hi + a_hi b_lo + a_hi b_hi``, the chunks summed, then ``+ bias``, then ``+ c``.

The products of TF32 parts are exact in float64 and every sum here is float64, so ``gemm_3xtf32``
returns the exact value of the 3xTF32 formula with ``lo`` kept exact; a tensor-core implementation
differs from it by the FP32 rounding of its accumulations (bounded per 64-wide chunk) and by reading
``lo`` at TF32 precision (at most 2^-22 of a product's magnitude). Pinned to the reference's own kernels:
``tests/golden/make_golden.py`` runs ``_split_kernel`` and ``_wide_gemm_persistent`` / ``_wide_gemm_tiles``
under the Triton interpreter (their one PTX instruction, ``cvt.rna.tf32.f32``, replaced by its bit
definition, which the known answers of the CPU tests pin), and this restatement equals those outputs: the
split bitwise, the products within 2e-7 of ``sum |x||w|`` (the interpreter's FP32 dots) on five shapes
(K 64 to 448, a partial last chunk, bias, accumulate, the input-gradient orientation).
"""
from __future__ import annotations

import numpy as np


def rna_tf32(x: np.ndarray) -> np.ndarray:
    """float32 -> float32 rounded to TF32, nearest with ties away from zero (finite inputs)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    sign = u & np.uint32(0x80000000)
    mag = u & np.uint32(0x7FFFFFFF)
    finite = mag < np.uint32(0x7F800000)
    rounded = (mag + np.uint32(0x1000)) & np.uint32(0xFFFFE000)  # half of the dropped 13 bits, then truncate
    out = np.where(finite, sign | rounded, u).astype(np.uint32)
    return out.view(np.float32)


def split(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(hi, lo) with hi = rna_tf32(x) and lo = x - hi in float32 (exact)."""
    x = np.asarray(x, dtype=np.float32)
    hi = rna_tf32(x)
    return hi, (x - hi).astype(np.float32)


def gemm_3xtf32(x: np.ndarray, w: np.ndarray, bias=None, c=None, chunk: int = 64) -> np.ndarray:
    """The 3xTF32 value of ``x @ w.T (+ bias) (+ c)`` for x [m, k], w [n, k], in float64."""
    xh, xl = (p.astype(np.float64) for p in split(x))
    wh, wl = (p.astype(np.float64) for p in split(w))
    m, k = x.shape
    acc = np.zeros((m, w.shape[0]), dtype=np.float64)
    for k0 in range(0, k, chunk):
        s = slice(k0, min(k0 + chunk, k))
        acc += xl[:, s] @ wh[:, s].T + xh[:, s] @ wl[:, s].T + xh[:, s] @ wh[:, s].T
    if bias is not None:
        acc += np.asarray(bias, dtype=np.float64)[None, :]
    if c is not None:
        acc += np.asarray(c, dtype=np.float64)
    return acc


def error_scale(x: np.ndarray, w: np.ndarray, bias=None, c=None) -> np.ndarray:
    """sum_k |x||w| (+ |bias| + |c|) per output: the scale FP32 accumulation errors are relative to."""
    s = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    if bias is not None:
        s += np.abs(np.asarray(bias, dtype=np.float64))[None, :]
    if c is not None:
        s += np.abs(np.asarray(c, dtype=np.float64))
    return s
