// The fused GatedMLP epilogue of MatRIS (fastmd/models/matris/op/triton_gated_ln.py):
//
//   out = silu(LN(core_x + core_lb)) * sigmoid(LN(gate_x + gate_lb)) (+ residual * res_weight)
//
// per row of width D in FP32 with LN(x) = (x - mean) rstd w + b, rstd = 1 / sqrt(var + eps),
// and its backward from the saved per-row mean / rstd (:57, :127; the 2-D tile variants :205,
// :280 apply the same formulas). One warp per row; lane l owns columns l + 32 i, the row sums
// are warp shuffle trees (fixed order: deterministic). Compiled without FMA contraction, so
// each product and sum rounds as in the reference's FP32 program (only the order of the row
// sums differs). The column sums of the linear biases' gradients are a two-pass fixed-order
// reduction (fmd_column_sum).

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kRowsPerCta = 8;
constexpr int kThreads = 32 * kRowsPerCta;

struct GlnArgs {
    const float* cx;
    const float* gx;
    const float* clb;
    const float* glb;
    const float* cw;
    const float* cb;
    const float* gw;
    const float* gb;
    const float* residual;
    const float* res_weight;
    const float* grad;  // backward only
    int64_t rows;
    int d;
    float eps_c, eps_g;
    float* out;         // forward: out; backward: grad_core_x
    float* out2;        // backward: grad_gate_x
    float* out3;        // backward: grad_residual (or null)
    float* cmean;
    float* crstd;
    float* gmean;
    float* grstd;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

template <int CPL>
__global__ void __launch_bounds__(kThreads) gated_ln_fwd_kernel(GlnArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    const float fd = float(a.d);
    float xc[CPL], xg[CPL];
    float sc = 0.f, sg = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = lane + 32 * i;
        const bool in = c < a.d;
        xc[i] = in ? __ldg(a.cx + row * a.d + c) : 0.f;
        xg[i] = in ? __ldg(a.gx + row * a.d + c) : 0.f;
        if (in && a.clb != nullptr) {
            xc[i] = xc[i] + __ldg(a.clb + c);
            xg[i] = xg[i] + __ldg(a.glb + c);
        }
        sc += xc[i];
        sg += xg[i];
    }
    const float cmu = warp_sum(sc) / fd, gmu = warp_sum(sg) / fd;
    float vc = 0.f, vg = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const bool in = lane + 32 * i < a.d;
        xc[i] = in ? xc[i] - cmu : 0.f;
        xg[i] = in ? xg[i] - gmu : 0.f;
        vc += xc[i] * xc[i];
        vg += xg[i] * xg[i];
    }
    const float crs = 1.0f / sqrtf(warp_sum(vc) / fd + a.eps_c);
    const float grs = 1.0f / sqrtf(warp_sum(vg) / fd + a.eps_g);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = lane + 32 * i;
        if (c >= a.d) continue;
        const float cy = xc[i] * crs * __ldg(a.cw + c) + __ldg(a.cb + c);
        const float gy = xg[i] * grs * __ldg(a.gw + c) + __ldg(a.gb + c);
        float r = (cy * sigmoid(cy)) * sigmoid(gy);
        if (a.residual != nullptr) r = r + __ldg(a.residual + row * a.d + c) * __ldg(a.res_weight + c);
        a.out[row * a.d + c] = r;
    }
    if (lane == 0) {
        a.cmean[row] = cmu;
        a.crstd[row] = crs;
        a.gmean[row] = gmu;
        a.grstd[row] = grs;
    }
}

template <int CPL>
__global__ void __launch_bounds__(kThreads) gated_ln_bwd_kernel(GlnArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    const float fd = float(a.d);
    const float cmu = a.cmean[row], crs = a.crstd[row], gmu = a.gmean[row], grs = a.grstd[row];
    float dxc[CPL], dxg[CPL], xhc[CPL], xhg[CPL];
    float s1c = 0.f, s2c = 0.f, s1g = 0.f, s2g = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = lane + 32 * i;
        dxc[i] = dxg[i] = xhc[i] = xhg[i] = 0.f;
        if (c >= a.d) continue;
        float xc = __ldg(a.cx + row * a.d + c), xg = __ldg(a.gx + row * a.d + c);
        if (a.clb != nullptr) {
            xc = xc + __ldg(a.clb + c);
            xg = xg + __ldg(a.glb + c);
        }
        const float cw = __ldg(a.cw + c), gw = __ldg(a.gw + c);
        const float g = __ldg(a.grad + row * a.d + c);
        xhc[i] = (xc - cmu) * crs;
        const float cy = xhc[i] * cw + __ldg(a.cb + c);
        const float cs = sigmoid(cy);
        const float core = cy * cs;
        xhg[i] = (xg - gmu) * grs;
        const float gy = xhg[i] * gw + __ldg(a.gb + c);
        const float gate = sigmoid(gy);
        const float d_cy = g * gate * (cs * (1.0f + cy * (1.0f - cs)));
        const float d_gy = g * core * (gate * (1.0f - gate));
        dxc[i] = d_cy * cw;
        dxg[i] = d_gy * gw;
        s1c += dxc[i];
        s2c += dxc[i] * xhc[i];
        s1g += dxg[i];
        s2g += dxg[i] * xhg[i];
        if (a.out3 != nullptr) a.out3[row * a.d + c] = g * __ldg(a.res_weight + c);
    }
    const float m1c = warp_sum(s1c) / fd, m2c = warp_sum(s2c) / fd;
    const float m1g = warp_sum(s1g) / fd, m2g = warp_sum(s2g) / fd;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = lane + 32 * i;
        if (c >= a.d) continue;
        a.out[row * a.d + c] = (dxc[i] - m1c - xhc[i] * m2c) * crs;
        a.out2[row * a.d + c] = (dxg[i] - m1g - xhg[i] * m2g) * grs;
    }
}

constexpr int kColRows = 128;  // rows per partial of the column sum

__global__ void column_partial_kernel(const float* __restrict__ x, int64_t rows, int cols, int64_t ld,
                                      float* __restrict__ partial) {
    const int64_t r0 = int64_t(blockIdx.x) * kColRows;
    const int64_t r1 = r0 + kColRows < rows ? r0 + kColRows : rows;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float s = 0.f;
        for (int64_t r = r0; r < r1; ++r) s += x[r * ld + c];
        partial[int64_t(blockIdx.x) * cols + c] = s;
    }
}

__global__ void column_final_kernel(const float* __restrict__ partial, int64_t n_partial, int cols,
                                    float* __restrict__ out) {
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int64_t b = 0; b < n_partial; ++b) s += partial[b * cols + c];
        out[c] = s;
    }
}


fmd_status launch_gln(GlnArgs& a, bool backward, cudaStream_t s) {
    const int64_t blocks = (a.rows + kRowsPerCta - 1) / kRowsPerCta;
    if (blocks > INT32_MAX) return FMD_ERR_UNSUPPORTED;
    const int cpl = (a.d + 31) / 32;
#define FMD_GLN(CPL)                                                                       \
    do {                                                                                   \
        if (backward)                                                                      \
            gated_ln_bwd_kernel<CPL><<<int(blocks), kThreads, 0, s>>>(a);                  \
        else                                                                               \
            gated_ln_fwd_kernel<CPL><<<int(blocks), kThreads, 0, s>>>(a);                  \
    } while (0)
    if (cpl <= 1) FMD_GLN(1);
    else if (cpl <= 2) FMD_GLN(2);
    else if (cpl <= 4) FMD_GLN(4);
    else if (cpl <= 8) FMD_GLN(8);
    else return FMD_ERR_UNSUPPORTED;
#undef FMD_GLN
    return check_launch();
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_gated_ln(const float* core_x, const float* gate_x, const float* core_lb, const float* gate_lb,
                        const float* core_w, const float* core_b, const float* gate_w, const float* gate_b,
                        const float* residual, const float* res_weight, int64_t rows, int32_t dim, float eps_core,
                        float eps_gate, float* out, float* core_mean, float* core_rstd, float* gate_mean,
                        float* gate_rstd, void* stream) {
    if (rows < 0 || dim < 1 || ((core_lb == nullptr) != (gate_lb == nullptr)) ||
        ((residual == nullptr) != (res_weight == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    if (core_x == nullptr || gate_x == nullptr || core_w == nullptr || core_b == nullptr || gate_w == nullptr ||
        gate_b == nullptr || out == nullptr || core_mean == nullptr || core_rstd == nullptr || gate_mean == nullptr ||
        gate_rstd == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    GlnArgs a{core_x, gate_x, core_lb, gate_lb, core_w, core_b, gate_w, gate_b, residual, res_weight, nullptr,
              rows, dim, eps_core, eps_gate, out, nullptr, nullptr, core_mean, core_rstd, gate_mean, gate_rstd};
    return launch_gln(a, false, as_stream(stream));
}

fmd_status fmd_gated_ln_bwd(const float* core_x, const float* gate_x, const float* core_lb, const float* gate_lb,
                            const float* core_w, const float* core_b, const float* gate_w, const float* gate_b,
                            const float* res_weight, const float* grad_out, const float* core_mean,
                            const float* core_rstd, const float* gate_mean, const float* gate_rstd, int64_t rows,
                            int32_t dim, float* grad_core_x, float* grad_gate_x, float* grad_residual,
                            void* stream) {
    if (rows < 0 || dim < 1 || ((core_lb == nullptr) != (gate_lb == nullptr)) ||
        (grad_residual != nullptr && res_weight == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    if (core_x == nullptr || gate_x == nullptr || core_w == nullptr || core_b == nullptr || gate_w == nullptr ||
        gate_b == nullptr || grad_out == nullptr || core_mean == nullptr || core_rstd == nullptr ||
        gate_mean == nullptr || gate_rstd == nullptr || grad_core_x == nullptr || grad_gate_x == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    GlnArgs a{core_x, gate_x, core_lb, gate_lb, core_w, core_b, gate_w, gate_b, nullptr, res_weight, grad_out,
              rows, dim, 0.f, 0.f, grad_core_x, grad_gate_x, grad_residual, const_cast<float*>(core_mean),
              const_cast<float*>(core_rstd), const_cast<float*>(gate_mean), const_cast<float*>(gate_rstd)};
    return launch_gln(a, true, as_stream(stream));
}

fmd_status fmd_column_sum_workspace_bytes(int64_t rows, int32_t cols, size_t* bytes) {
    if (bytes == nullptr || rows < 0 || cols < 1) return FMD_ERR_INVALID_ARGUMENT;
    const int64_t n_partial = (rows + kColRows - 1) / kColRows;
    *bytes = size_t(n_partial > 0 ? n_partial : 1) * size_t(cols) * sizeof(float);
    return FMD_OK;
}

fmd_status fmd_column_sum(const float* x, int64_t rows, int32_t cols, int64_t ld, void* workspace,
                          size_t workspace_bytes, float* out, void* stream) {
    if (rows < 0 || cols < 1 || ld < cols || out == nullptr || (rows > 0 && x == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    fmd_column_sum_workspace_bytes(rows, cols, &need);
    if (workspace == nullptr || workspace_bytes < need) return FMD_ERR_WORKSPACE;
    const int64_t n_partial = (rows + kColRows - 1) / kColRows;
    cudaStream_t s = as_stream(stream);
    float* partial = static_cast<float*>(workspace);
    if (n_partial == 0) {
        cudaError_t err = cudaMemsetAsync(out, 0, sizeof(float) * size_t(cols), s);
        return err == cudaSuccess ? FMD_OK : record_cuda_error(err);
    }
    if (n_partial > INT32_MAX) return FMD_ERR_UNSUPPORTED;
    const int threads = cols < 256 ? ((cols + 31) / 32) * 32 : 256;
    column_partial_kernel<<<int(n_partial), threads, 0, s>>>(x, rows, cols, ld, partial);
    column_final_kernel<<<(cols + 255) / 256, 256, 0, s>>>(partial, n_partial, cols, out);
    return check_launch();
}

}  // extern "C"
