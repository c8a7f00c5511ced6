// Residual add of the MatRIS interaction blocks with a frozen per-column weight.
//
//   op 0  forward   out[r, c] = delta[r, c] + residual[r, c] * weight[c]
//   op 1  backward  out[r, c] = gout[r, c] * weight[c]          (grad of residual; grad of delta is gout)
//
// (fastmd/models/matris/op/triton_residual_add.py:40 _residual_add_fwd, :64
// _residual_add_bwd). The product is rounded before the addition (no FMA
// contraction: __fmul_rn then __fadd_rn), the operation order of the
// reference run by the Triton interpreter, so the result is bit-identical to
// it. Each operand keeps its own row stride (a column view of a wider buffer
// is read in place). Pure streaming, HBM-bound: 12 bytes per element moved
// (forward), 8 bytes (backward); one thread per 4 consecutive columns with
// 16-byte accesses where widths, strides and pointers allow, else one thread
// per column; the weight row stays in L1/L2.

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float axpy_rn(float d, float r, float w) { return __fadd_rn(d, __fmul_rn(r, w)); }

template <int OP, bool VEC4>
__global__ void __launch_bounds__(kThreads)
    residual_add_kernel(const float* __restrict__ delta, int64_t ldd, const float* __restrict__ residual, int64_t ldr,
                        const float* __restrict__ weight, int64_t rows, int dim, float* __restrict__ out,
                        int64_t ldo) {
    constexpr int V = VEC4 ? 4 : 1;
    const int groups = dim / V;
    const int64_t total = rows * groups;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / groups;
        const int c = int(t - r * groups) * V;
        if constexpr (VEC4) {
            const float4 w = ldg4(weight + c);
            const float4 x = ldg4(residual + r * ldr + c);
            float4 y;
            if constexpr (OP == 0) {
                const float4 d = ldg4(delta + r * ldd + c);
                y = make_float4(axpy_rn(d.x, x.x, w.x), axpy_rn(d.y, x.y, w.y), axpy_rn(d.z, x.z, w.z),
                                axpy_rn(d.w, x.w, w.w));
            } else {
                y = make_float4(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y), __fmul_rn(x.z, w.z), __fmul_rn(x.w, w.w));
            }
            st4(out + r * ldo + c, y);
        } else {
            const float w = __ldg(weight + c), x = __ldg(residual + r * ldr + c);
            out[r * ldo + c] = OP == 0 ? axpy_rn(__ldg(delta + r * ldd + c), x, w) : __fmul_rn(x, w);
        }
    }
}

template <int OP>
void launch(bool vec4, const float* delta, int64_t ldd, const float* residual, int64_t ldr, const float* weight,
            int64_t rows, int dim, float* out, int64_t ldo, cudaStream_t s) {
    if (vec4) {
        residual_add_kernel<OP, true><<<grid_for(rows * (dim / 4), kThreads), kThreads, 0, s>>>(
            delta, ldd, residual, ldr, weight, rows, dim, out, ldo);
    } else {
        residual_add_kernel<OP, false><<<grid_for(rows * dim, kThreads), kThreads, 0, s>>>(delta, ldd, residual, ldr,
                                                                                          weight, rows, dim, out, ldo);
    }
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_residual_add(int32_t op, const float* delta, int64_t ldd, const float* residual, int64_t ldr,
                            const float* weight, int64_t rows, int32_t dim, float* out, int64_t ldo, void* stream) {
    if ((op != 0 && op != 1) || rows < 0 || dim < 1 || ldr < dim || ldo < dim || (op == 0 && ldd < dim))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    if (residual == nullptr || weight == nullptr || out == nullptr || (op == 0 && delta == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    const bool vec4 = dim % 4 == 0 && ldr % 4 == 0 && ldo % 4 == 0 && aligned16(residual) && aligned16(weight) &&
                      aligned16(out) && (op == 1 || (ldd % 4 == 0 && aligned16(delta)));
    const cudaStream_t s = as_stream(stream);
    if (op == 0)
        launch<0>(vec4, delta, ldd, residual, ldr, weight, rows, dim, out, ldo, s);
    else
        launch<1>(vec4, delta, ldd, residual, ldr, weight, rows, dim, out, ldo, s);
    return check_launch();
}

}  // extern "C"
