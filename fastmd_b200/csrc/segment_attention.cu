// Segment attention (the MatRIS receiver softmax-weighted sum) over a CSR:
//
//   out[s, d] = sum_{rows i of segment s} softmax_d(logits[i, d] over s) * value[i, d]
//
// The reference's kernels (fastmd/models/matris/op/triton_segment_attention.py):
// forward :62 and backward :128 one program per segment, the paired forward
// :210 (two CSRs sharing the values) and the paired row backward :319.
//
// One warp per segment, 8 segments per 256-thread CTA; lane l owns columns
// c0 + l + 32 i (i < CPL) of each 32*CPL-wide column block, so every load of a
// row is a coalesced 128-byte line per i. The rows of a segment are visited in
// CSR order with the reference's online recurrence (m' = max(m, l); denom and
// acc rescaled by e^(m - m'), plus e^(l - m') and e^(l - m') v), the next rows'
// logits and values loaded ahead of the sequential update. Compiled without
// FMA contraction: each operation rounds as in the reference's FP32 program.
// perm == null is the identity CSR (row = j). Rows outside [0, rows) in perm
// or segments outside [0, num_segment) raise FMD_FLAG_INDEX_RANGE and are
// skipped.

#include "common.cuh"

namespace fmd {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kAhead = 4;  // rows loaded ahead of the recurrence

struct SegAttnArgs {
    const float* logits;
    int64_t ldl;
    const float* value;
    int64_t ldv;
    const int64_t* perm;
    const int64_t* off;
    int64_t rows, num_segment, skip;
    int dim;
    float* out;        // [S, dim]
    float* lse;        // [S, dim] or null
    float* seg_max;    // [S, dim] or null
    float* seg_denom;  // [S, dim] or null
    int32_t* flags;
};

__device__ __forceinline__ int64_t row_of(const int64_t* perm, int64_t j, int64_t rows, int32_t* flags, bool& ok) {
    const int64_t r = perm != nullptr ? __ldg(perm + j) : j;
    ok = r >= 0 && r < rows;
    if (!ok) raise_flag(flags, FMD_FLAG_INDEX_RANGE);
    return r;
}

template <int CPL>
__global__ void __launch_bounds__(kThreads) segattn_fwd_kernel(SegAttnArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t s = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    if (s >= a.num_segment) return;
    const int64_t start = __ldg(a.off + s);
    const int64_t end = s == a.skip ? start : __ldg(a.off + s + 1);
    for (int c0 = 0; c0 < a.dim; c0 += 32 * CPL) {
        float m[CPL], denom[CPL], acc[CPL];
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            m[i] = -INFINITY;
            denom[i] = 0.0f;
            acc[i] = 0.0f;
        }
        for (int64_t j0 = start; j0 < end; j0 += kAhead) {
            float lg[kAhead][CPL], vl[kAhead][CPL];
            bool live[kAhead];
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                live[u] = j0 + u < end;
                int64_t r = 0;
                if (live[u]) r = row_of(a.perm, j0 + u, a.rows, a.flags, live[u]);
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const int c = c0 + lane + 32 * i;
                    const bool in = live[u] && c < a.dim;
                    lg[u][i] = in ? __ldg(a.logits + r * a.ldl + c) : -INFINITY;
                    vl[u][i] = in ? __ldg(a.value + r * a.ldv + c) : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                if (!live[u]) continue;
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const float m_new = fmaxf(m[i], lg[u][i]);
                    const float old_scale = expf(m[i] - m_new);
                    const float new_scale = expf(lg[u][i] - m_new);
                    denom[i] = denom[i] * old_scale + new_scale;
                    acc[i] = acc[i] * old_scale + new_scale * vl[u][i];
                    m[i] = m_new;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = c0 + lane + 32 * i;
            if (c >= a.dim) continue;
            const int64_t o = s * a.dim + c;
            a.out[o] = denom[i] > 0.0f ? acc[i] / denom[i] : 0.0f;
            if (a.lse != nullptr) a.lse[o] = denom[i] > 0.0f ? m[i] + logf(denom[i]) : -INFINITY;
            if (a.seg_max != nullptr) a.seg_max[o] = m[i];
            if (a.seg_denom != nullptr) a.seg_denom[o] = denom[i];
        }
    }
}

struct SegAttnBwdArgs {
    const float* logits;
    int64_t ldl;
    const float* value;
    int64_t ldv;
    const float* out;   // [S, dim]
    const float* gout;  // [S, dim]
    const float* glse;  // [S, dim] or null
    const int64_t* perm;
    const int64_t* off;
    int64_t rows, num_segment, skip;
    int dim;
    float* grad_logits;
    int64_t ldgl;
    float* grad_value;
    int64_t ldgv;
    int32_t* flags;
};

template <int CPL>
__global__ void __launch_bounds__(kThreads) segattn_bwd_kernel(SegAttnBwdArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t s = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    if (s >= a.num_segment) return;
    const int64_t start = __ldg(a.off + s);
    const int64_t end = s == a.skip ? start : __ldg(a.off + s + 1);
    for (int c0 = 0; c0 < a.dim; c0 += 32 * CPL) {
        float m[CPL], denom[CPL];
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            m[i] = -INFINITY;
            denom[i] = 0.0f;
        }
        for (int64_t j0 = start; j0 < end; j0 += kAhead) {
            float lg[kAhead][CPL];
            bool live[kAhead];
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                live[u] = j0 + u < end;
                int64_t r = 0;
                if (live[u]) r = row_of(a.perm, j0 + u, a.rows, nullptr, live[u]);
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const int c = c0 + lane + 32 * i;
                    lg[u][i] = (live[u] && c < a.dim) ? __ldg(a.logits + r * a.ldl + c) : -INFINITY;
                }
            }
#pragma unroll
            for (int u = 0; u < kAhead; ++u) {
                if (!live[u]) continue;
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const float m_new = fmaxf(m[i], lg[u][i]);
                    denom[i] = denom[i] * expf(m[i] - m_new) + expf(lg[u][i] - m_new);
                    m[i] = m_new;
                }
            }
        }
        float inv[CPL], go[CPL], os[CPL], gl[CPL];
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = c0 + lane + 32 * i;
            const bool in = c < a.dim;
            inv[i] = denom[i] > 0.0f ? 1.0f / denom[i] : 0.0f;
            go[i] = in ? __ldg(a.gout + s * a.dim + c) : 0.0f;
            os[i] = in ? __ldg(a.out + s * a.dim + c) : 0.0f;
            gl[i] = (in && a.glse != nullptr) ? __ldg(a.glse + s * a.dim + c) : 0.0f;
        }
        for (int64_t j = start; j < end; ++j) {
            bool ok;
            const int64_t r = row_of(a.perm, j, a.rows, a.flags, ok);
            if (!ok) continue;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = c0 + lane + 32 * i;
                if (c >= a.dim) continue;
                const float logit = __ldg(a.logits + r * a.ldl + c);
                const float val = __ldg(a.value + r * a.ldv + c);
                const float alpha = expf(logit - m[i]) * inv[i];
                a.grad_value[r * a.ldgv + c] = alpha * go[i];
                float g = alpha * go[i] * (val - os[i]);
                if (a.glse != nullptr) g = g + alpha * gl[i];
                a.grad_logits[r * a.ldgl + c] = g;
            }
        }
    }
}

struct PairedBwdArgs {
    const float* logits_a;
    int64_t ldla;
    const float* logits_b;
    int64_t ldlb;
    const float* value;
    int64_t ldv;
    const float* gout_a;
    const float* gout_b;
    const float* out_a;
    const float* out_b;
    const float* max_a;
    const float* denom_a;
    const float* max_b;
    const float* denom_b;
    const int64_t* segment_a;
    const int64_t* segment_b;
    const float* glse_a;  // or null (then glse_b is null too)
    const float* glse_b;
    int64_t rows, num_segment, skip;
    int dim;
    float* grad_logits_a;
    int64_t ldga;
    float* grad_logits_b;
    int64_t ldgb;
    float* grad_value;  // [rows, dim]
    int32_t* flags;
};

// One thread per (row, column); the per-segment statistics are gathered by
// the row's two segment ids. A skipped segment's side contributes exactly 0.
__global__ void __launch_bounds__(kThreads) paired_bwd_rows_kernel(PairedBwdArgs a) {
    const int64_t total = a.rows * a.dim;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = t / a.dim;
        const int c = int(t - r * a.dim);
        const int64_t sa = __ldg(a.segment_a + r), sb = __ldg(a.segment_b + r);
        if (sa < 0 || sa >= a.num_segment || sb < 0 || sb >= a.num_segment) {
            raise_flag(a.flags, FMD_FLAG_INDEX_RANGE);
            continue;
        }
        const int64_t oa = sa * a.dim + c, ob = sb * a.dim + c;
        const float la = __ldg(a.logits_a + r * a.ldla + c), lb = __ldg(a.logits_b + r * a.ldlb + c);
        const float val = __ldg(a.value + r * a.ldv + c);
        const float da = __ldg(a.denom_a + oa), db = __ldg(a.denom_b + ob);
        const float alpha_a = expf(la - __ldg(a.max_a + oa)) * (da > 0.0f ? 1.0f / da : 0.0f);
        const float alpha_b = expf(lb - __ldg(a.max_b + ob)) * (db > 0.0f ? 1.0f / db : 0.0f);
        const bool live_a = sa != a.skip, live_b = sb != a.skip;
        const float term_a = live_a ? alpha_a * __ldg(a.gout_a + oa) : 0.0f;
        const float term_b = live_b ? alpha_b * __ldg(a.gout_b + ob) : 0.0f;
        float ga = term_a * (val - __ldg(a.out_a + oa));
        float gb = term_b * (val - __ldg(a.out_b + ob));
        if (a.glse_a != nullptr) {
            ga = ga + alpha_a * __ldg(a.glse_a + oa);
            gb = gb + alpha_b * __ldg(a.glse_b + ob);
        }
        a.grad_logits_a[r * a.ldga + c] = live_a ? ga : 0.0f;
        a.grad_logits_b[r * a.ldgb + c] = live_b ? gb : 0.0f;
        a.grad_value[r * a.dim + c] = term_a + term_b;
    }
}

int cpl_for(int dim) { return dim <= 32 ? 1 : dim <= 64 ? 2 : 4; }

}  // namespace
}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_segment_attention(const float* logits, int64_t ldl, const float* value, int64_t ldv,
                                 const int64_t* perm, const int64_t* off, int64_t rows, int64_t num_segment,
                                 int32_t dim, int64_t skip_segment, float* out, float* lse, float* seg_max,
                                 float* seg_denom, int32_t* flags, void* stream) {
    if (num_segment < 0 || rows < 0 || dim < 1 || ldl < dim || ldv < dim || (skip_segment != -1 && (skip_segment < 0 || skip_segment >= num_segment)) || (num_segment > 0 && (off == nullptr || out == nullptr)) ||
        (rows > 0 && (logits == nullptr || value == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    if (num_segment == 0) return FMD_OK;
    SegAttnArgs a{logits, ldl, value, ldv, perm, off, rows, num_segment, skip_segment, dim,
                  out, lse, seg_max, seg_denom, flags};
    const int64_t blocks = (num_segment + kWarps - 1) / kWarps;
    if (blocks > INT32_MAX) return FMD_ERR_UNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    switch (cpl_for(dim)) {
        case 1: segattn_fwd_kernel<1><<<int(blocks), kThreads, 0, st>>>(a); break;
        case 2: segattn_fwd_kernel<2><<<int(blocks), kThreads, 0, st>>>(a); break;
        default: segattn_fwd_kernel<4><<<int(blocks), kThreads, 0, st>>>(a); break;
    }
    return check_launch();
}

fmd_status fmd_segment_attention_bwd(const float* logits, int64_t ldl, const float* value, int64_t ldv,
                                     const float* out, const float* gout, const float* glse, const int64_t* perm,
                                     const int64_t* off, int64_t rows, int64_t num_segment, int32_t dim,
                                     int64_t skip_segment, float* grad_logits, int64_t ldgl, float* grad_value,
                                     int64_t ldgv, int32_t* flags, void* stream) {
    if (num_segment < 0 || rows < 0 || dim < 1 || ldl < dim || ldv < dim || ldgl < dim || ldgv < dim ||
        (skip_segment != -1 && (skip_segment < 0 || skip_segment >= num_segment)) ||
        (num_segment > 0 && (off == nullptr || out == nullptr || gout == nullptr)) ||
        (rows > 0 && (logits == nullptr || value == nullptr || grad_logits == nullptr || grad_value == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    if (num_segment == 0) return FMD_OK;
    SegAttnBwdArgs a{logits, ldl, value, ldv, out, gout, glse, perm, off, rows, num_segment, skip_segment, dim,
                     grad_logits, ldgl, grad_value, ldgv, flags};
    const int64_t blocks = (num_segment + kWarps - 1) / kWarps;
    if (blocks > INT32_MAX) return FMD_ERR_UNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    switch (cpl_for(dim)) {
        case 1: segattn_bwd_kernel<1><<<int(blocks), kThreads, 0, st>>>(a); break;
        case 2: segattn_bwd_kernel<2><<<int(blocks), kThreads, 0, st>>>(a); break;
        default: segattn_bwd_kernel<4><<<int(blocks), kThreads, 0, st>>>(a); break;
    }
    return check_launch();
}

fmd_status fmd_paired_segment_attention_bwd_rows(
    const float* logits_a, int64_t ldla, const float* logits_b, int64_t ldlb, const float* value, int64_t ldv,
    const float* gout_a, const float* gout_b, const float* out_a, const float* out_b, const float* max_a,
    const float* denom_a, const float* max_b, const float* denom_b, const int64_t* segment_a,
    const int64_t* segment_b, const float* glse_a, const float* glse_b, int64_t rows, int64_t num_segment,
    int32_t dim, int64_t skip_segment, float* grad_logits_a, int64_t ldga, float* grad_logits_b, int64_t ldgb,
    float* grad_value, int32_t* flags, void* stream) {
    if (rows < 0 || num_segment < 0 || dim < 1 || ldla < dim || ldlb < dim || ldv < dim || ldga < dim ||
        ldgb < dim || (skip_segment != -1 && (skip_segment < 0 || skip_segment >= num_segment)) ||
        ((glse_a == nullptr) != (glse_b == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    if (logits_a == nullptr || logits_b == nullptr || value == nullptr || gout_a == nullptr || gout_b == nullptr ||
        out_a == nullptr || out_b == nullptr || max_a == nullptr || denom_a == nullptr || max_b == nullptr ||
        denom_b == nullptr || segment_a == nullptr || segment_b == nullptr || grad_logits_a == nullptr ||
        grad_logits_b == nullptr || grad_value == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    PairedBwdArgs a{logits_a, ldla, logits_b, ldlb, value, ldv, gout_a, gout_b, out_a, out_b, max_a, denom_a,
                    max_b, denom_b, segment_a, segment_b, glse_a, glse_b, rows, num_segment, skip_segment, dim,
                    grad_logits_a, ldga, grad_logits_b, ldgb, grad_value, flags};
    paired_bwd_rows_kernel<<<grid_for(rows * dim, kThreads), kThreads, 0, as_stream(stream)>>>(a);
    return check_launch();
}

}  // extern "C"
