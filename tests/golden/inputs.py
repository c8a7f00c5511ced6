"""Seeded FP32 inputs that need no stored copy: a SplitMix64 counter stream (plain uint64 arithmetic,
the same on every platform and NumPy version), so a fixture can keep only the reference's outputs and
the test regenerates the inputs. Test infrastructure only."""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def counter_floats(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """float32 values uniform on [-scale, scale) with 24 significant bits, element i from the SplitMix64
    output of counter i of stream ``seed``."""
    n = int(np.prod(shape))
    with np.errstate(over="ignore"):
        z = (np.arange(n, dtype=np.uint64) + np.uint64(1)) * _GOLDEN + np.uint64(seed) * _M2
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    u = (z >> np.uint64(40)).astype(np.float64) / float(1 << 24)  # 24 bits: exact in float32
    return ((2.0 * u - 1.0) * scale).astype(np.float32).reshape(shape)


# Wide-GEMM fixture cases, (rows, K, N, transposed, bias, c): the config-2 first layer (K 264, a partial
# last 64-wide chunk), an input gradient dX = dY W (B = W, K-major W^T) into c, the accumulate form, a
# 64-wide tile, and K >= 384 (the reference's per-tile kernel); each one full 128-row tile and a ragged tail.
WIDE_GEMM_CASES = {"k264_n256_bias": (130, 264, 256, False, True, False),
                   "grad_k256_n128": (131, 256, 128, True, False, True),
                   "k128_n128_c": (133, 128, 128, False, False, True),
                   "k64_n64_bias": (150, 64, 64, False, True, False),
                   "k448_n64_bias": (129, 448, 64, False, True, False)}


def wide_gemm_inputs(i, m, k, n, transposed, has_bias, has_c):
    """The inputs of wide-GEMM case ``i``: a [m, k], w [n, k] (or [k, n] for the input-gradient form),
    bias [n], c [m, n], from counter streams 4i .. 4i + 3."""
    a = counter_floats(4 * i, (m, k), 1.7)
    w = counter_floats(4 * i + 1, (k, n) if transposed else (n, k), 1.7 / float(np.sqrt(k)))
    bias = counter_floats(4 * i + 2, (n,), 1.0) if has_bias else None
    c = counter_floats(4 * i + 3, (m, n), 1.0) if has_c else None
    return a, w, bias, c
