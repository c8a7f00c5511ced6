"""The definition of PTX ``cvt.rna.tf32.f32`` (round an FP32 value to TF32: nearest, ties away from
zero, the low 13 bits of the pattern cleared; NaN and infinities unchanged) as a Triton function the
interpreter can run. ``make_golden.py`` substitutes it for the reference wide GEMM's ``_rna_tf32``
(fastmd/engine/kernels/triton_wide_gemm.py:63), whose inline PTX the interpreter cannot execute.
Imported only after ``TRITON_INTERPRET=1`` is set."""
import triton
import triton.language as tl


@triton.jit
def rna_tf32(x):
    u = x.to(tl.uint32, bitcast=True)
    mag = u & 0x7FFFFFFF
    rounded = (u & 0x80000000) | ((mag + 0x1000) & 0xFFFFE000)
    return tl.where(mag < 0x7F800000, rounded, u).to(tl.float32, bitcast=True)
