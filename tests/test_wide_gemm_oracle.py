"""The 3xTF32 oracle on the CPU: TF32 rounding known answers (the PTX definition of
cvt.rna.tf32.f32: nearest, ties away from zero, 10 explicit mantissa bits), the exactness of the
hi/lo split, and the accuracy of the 3xTF32 formula against float64."""
import numpy as np

from oracle import wide_gemm as ow


def _f(v):
    return np.array(v, dtype=np.float32)


def test_rna_tf32_known_answers():
    cases = [
        (1.0, 1.0),
        (1 + 2.0**-12, 1.0),                      # below half an ulp: down
        (1 + 2.0**-11, 1 + 2.0**-10),             # exact tie: away from zero
        (1 + 2.0**-11 + 2.0**-23, 1 + 2.0**-10),  # above the tie: up
        (1 + 2.0**-10 + 2.0**-11, 1 + 2.0**-9),   # tie with an odd last bit: still away
        (-(1 + 2.0**-11), -(1 + 2.0**-10)),       # negative tie: away from zero
        (2 - 2.0**-23, 2.0),                      # carry into the exponent
        (3.0 * 2.0**-136, 3.0 * 2.0**-136),       # subnormal, pattern 0x6000: exact
        (0.0, 0.0),
    ]
    got = ow.rna_tf32(_f([a for a, _ in cases]))
    np.testing.assert_array_equal(got, _f([b for _, b in cases]))
    assert np.signbit(ow.rna_tf32(_f([-0.0])))[0]
    special = ow.rna_tf32(_f([np.inf, -np.inf, np.nan]))
    assert np.isposinf(special[0]) and np.isneginf(special[1]) and np.isnan(special[2])
    # 13 low bits zero for every finite input
    x = np.random.default_rng(0).standard_normal(10_000).astype(np.float32) * 1e3
    assert not np.any(ow.rna_tf32(x).view(np.uint32) & 0x1FFF)


def test_split_is_exact_and_small():
    x = (np.random.default_rng(1).standard_normal(50_000) * np.exp(np.random.default_rng(2).uniform(-20, 20, 50_000)))
    x = x.astype(np.float32)
    hi, lo = ow.split(x)
    np.testing.assert_array_equal(hi.astype(np.float64) + lo.astype(np.float64), x.astype(np.float64))
    assert np.all(np.abs(lo) <= np.abs(hi) * 2.0**-11 * (1 + 1e-7))


def test_3xtf32_formula_is_fp32_accurate():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 264)).astype(np.float32)
    w = (rng.standard_normal((96, 264)) / 16).astype(np.float32)
    b = rng.standard_normal(96).astype(np.float32)
    exact = x.astype(np.float64) @ w.astype(np.float64).T + b
    got = ow.gemm_3xtf32(x, w, bias=b)
    scale = ow.error_scale(x, w, bias=b)
    assert np.max(np.abs(got - exact) / scale) < 2.0**-20   # the dropped lo*lo term: < 2^-22 per product
    # one TF32 product alone is far coarser: the lo terms carry the FP32 accuracy
    one = ow.rna_tf32(x).astype(np.float64) @ ow.rna_tf32(w).astype(np.float64).T + b
    assert np.max(np.abs(one - exact) / scale) > 2.0**-14


def _golden_cases():
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(here))
    from inputs import WIDE_GEMM_CASES, wide_gemm_inputs

    return np.load(here / "wide_gemm.npz"), WIDE_GEMM_CASES, wide_gemm_inputs


def test_oracle_matches_the_reference_kernel():
    """The reference's own 3xTF32 kernels (_split_kernel, _wide_gemm_persistent / _wide_gemm_tiles of
    fastmd/engine/kernels/triton_wide_gemm.py, run by the Triton interpreter with cvt.rna.tf32.f32 as its
    bit definition; tests/golden/make_golden.py) against the oracle: the split bitwise, the products within
    FP32 rounding of the chunk sums (the interpreter's dots are FP32; the oracle's sums are exact)."""
    golden, cases, inputs = _golden_cases()
    for i, (tag, (m, k, n, transposed, has_bias, has_c)) in enumerate(cases.items()):
        a, w, bias, c = inputs(i, m, k, n, transposed, has_bias, has_c)
        assert list(golden[f"wg_{tag}_shape"]) == [m, k, n, transposed, has_bias, has_c]
        wk = np.ascontiguousarray(w.T if transposed else w)  # the [N, K] operand: y = a wk^T
        ref = ow.gemm_3xtf32(a, wk, bias=bias, c=c)
        scale = ow.error_scale(a, wk, bias=bias, c=c)
        err = np.abs(golden[f"wg_{tag}_y"].astype(np.float64) - ref) / scale
        assert err.max() < 5e-7, (tag, err.max())
        if f"wg_{tag}_hi" in golden:
            hi, lo = ow.split(wk)
            np.testing.assert_array_equal(golden[f"wg_{tag}_hi"], hi)
            np.testing.assert_array_equal(golden[f"wg_{tag}_lo"], lo)
