// The epilogue of the decomposed indexed-concat first layer (MatRIS GatedMLP on
// line-graph rows): the projections p_k = X_k W_k^T are computed on the source
// rows, then per output row
//
//   preact = p0[r] + p1[ia[r]] + p2[ib[r]] (+ p3[ic[r]]) + bias     [rows, 2H]
//   core_act = silu(preact[:, :H]),  gate_act = silu(preact[:, H:])
//
// with silu(x) = x * (1 / (1 + e^-x)), the additions in that order in FP32
// (fastmd/engine/kernels/decomposed_indexed_cat_silu_linear.py:97, :156).
// The backward's SiLU derivative d = g s (1 + x (1 - s)) per half (:234,
// :383) is written per row; its scatter into the gathered projections is the
// deterministic CSR row sum of fmd_gather_rows_bwd (no atomics). One thread
// per (row, column of a half); consecutive threads take consecutive columns.
// Compiled without FMA contraction (each operation rounds as in the reference).

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kMaxGathered = 3;
constexpr int kThreads = 256;

struct GasArgs {
    const float* p0;
    int64_t ldp0;
    const float* src[kMaxGathered];
    const int64_t* index[kMaxGathered];
    int64_t ld[kMaxGathered];
    int64_t n_src[kMaxGathered];
    int n_gathered;
    const float* bias;
    int64_t rows;
    int h;
    float* preact;
    float* core_act;
    float* gate_act;
    int32_t* flags;
};

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void __launch_bounds__(kThreads) gather_add_silu_kernel(GasArgs a) {
    const int64_t total = a.rows * a.h;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / a.h;
        const int c = int(t - r * a.h);
        float core = __ldg(a.p0 + r * a.ldp0 + c);
        float gate = __ldg(a.p0 + r * a.ldp0 + a.h + c);
        for (int k = 0; k < a.n_gathered; ++k) {
            const int64_t i = __ldg(a.index[k] + r);
            if (i < 0 || i >= a.n_src[k]) {  // out of range: contributes nothing, flagged
                raise_flag(a.flags, FMD_FLAG_INDEX_RANGE);
                continue;
            }
            core = core + __ldg(a.src[k] + i * a.ld[k] + c);
            gate = gate + __ldg(a.src[k] + i * a.ld[k] + a.h + c);
        }
        if (a.bias != nullptr) {
            core = core + __ldg(a.bias + c);
            gate = gate + __ldg(a.bias + a.h + c);
        }
        a.preact[r * 2 * a.h + c] = core;
        a.preact[r * 2 * a.h + a.h + c] = gate;
        a.core_act[r * a.h + c] = core * sigmoid(core);
        a.gate_act[r * a.h + c] = gate * sigmoid(gate);
    }
}

__global__ void __launch_bounds__(kThreads) silu_pair_bwd_kernel(const float* __restrict__ grad_core,
                                                                 const float* __restrict__ grad_gate,
                                                                 const float* __restrict__ preact, int64_t rows, int h,
                                                                 float* __restrict__ grad_pre, int64_t ldgp) {
    const int64_t total = rows * h;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / h;
        const int c = int(t - r * h);
        const float x0 = __ldg(preact + r * 2 * h + c), x1 = __ldg(preact + r * 2 * h + h + c);
        const float s0 = sigmoid(x0), s1 = sigmoid(x1);
        grad_pre[r * ldgp + c] = __ldg(grad_core + t) * s0 * (1.0f + x0 * (1.0f - s0));
        grad_pre[r * ldgp + h + c] = __ldg(grad_gate + t) * s1 * (1.0f + x1 * (1.0f - s1));
    }
}

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_gather_add_silu(const float* p0, int64_t ldp0, const fmd_cat_part* gathered, int32_t n_gathered,
                               const float* bias, int64_t rows, int32_t h, float* preact, float* core_act,
                               float* gate_act, int32_t* flags, void* stream) {
    if (rows < 0 || h < 1 || n_gathered < 0 || n_gathered > kMaxGathered || ldp0 < 2 * int64_t(h) ||
        (n_gathered > 0 && gathered == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    if (p0 == nullptr || preact == nullptr || core_act == nullptr || gate_act == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    GasArgs a{};
    a.p0 = p0;
    a.ldp0 = ldp0;
    for (int k = 0; k < n_gathered; ++k) {
        const fmd_cat_part& p = gathered[k];
        if (p.src == nullptr || p.index == nullptr || p.ld < 2 * int64_t(h) || p.n_src < 0)
            return FMD_ERR_INVALID_ARGUMENT;
        a.src[k] = p.src;
        a.index[k] = p.index;
        a.ld[k] = p.ld;
        a.n_src[k] = p.n_src;
    }
    a.n_gathered = n_gathered;
    a.bias = bias;
    a.rows = rows;
    a.h = h;
    a.preact = preact;
    a.core_act = core_act;
    a.gate_act = gate_act;
    a.flags = flags;
    gather_add_silu_kernel<<<grid_for(rows * h, kThreads), kThreads, 0, as_stream(stream)>>>(a);
    return check_launch();
}

fmd_status fmd_silu_pair_bwd(const float* grad_core, const float* grad_gate, const float* preact, int64_t rows,
                             int32_t h, float* grad_pre, int64_t ldgp, void* stream) {
    if (rows < 0 || h < 1 || ldgp < 2 * int64_t(h)) return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    if (grad_core == nullptr || grad_gate == nullptr || preact == nullptr || grad_pre == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    silu_pair_bwd_kernel<<<grid_for(rows * h, kThreads), kThreads, 0, as_stream(stream)>>>(grad_core, grad_gate,
                                                                                         preact, rows, h, grad_pre,
                                                                                         ldgp);
    return check_launch();
}

}  // extern "C"
