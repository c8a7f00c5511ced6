// IEEE FP32 GEMM on the CUDA cores: the parity path of the dense edge/node
// layers (TF32 off), for the small and latency-bound shapes of a 135-atom
// step where tensor-core tiles would sit mostly idle.
//
//   Y[M, N] (=|+=) act( A'[M, K] . op(W) + bias )
//   op(W) = W^T for W [N, K] (nn.Linear layout, trans_w = 1), W for W [K, N]
//   A' = A, or A * silu'(A_pre) elementwise when a_pre is given (the SiLU
//   backward of the previous layer fused into this GEMM's operand load)
//   act = identity or SiLU (the pre-activation optionally stored)
//
// 64x64 output tile per 256-thread CTA, 16-deep K slices staged in shared
// memory (double-buffered: the next slice's loads overlap the current slice's
// products), 4x4 outputs per thread; every output is one sequential FP32 FMA
// chain over K (deterministic, independent of the tiling of M and N).

#include "common.cuh"

namespace fmd {

constexpr int BM = 64, BN = 64, BK = 16;

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ float silu_grad(float x) {
    const float s = 1.0f / (1.0f + expf(-x));
    return s * (1.0f + x * (1.0f - s));
}

struct GemmArgs {
    const float* a;
    int64_t lda;
    const float* a_pre;   // optional: multiply A by silu'(a_pre)
    int64_t lda_pre;
    const float* w;
    int64_t ldw;
    int trans_w;
    const float* bias;    // [N] or null
    float* y;
    int64_t ldy;
    float* y_pre;         // optional pre-activation output
    int64_t ldy_pre;
    int64_t m;
    int n, k;
    int act;              // 0 identity, 1 SiLU
    int accumulate;
};

// the operand values of one K slice that thread t stages: A rows (t + 256 q) / 16, k (t + 256 q) % 16;
// W: columns (t + 256 q) / 16 and k % 16 (W [N, K]), or k (t + 256 q) / 64 and columns % 64 (W [K, N])
__device__ __forceinline__ void load_slice(const GemmArgs& g, int64_t row0, int col0, int k0, float (&pa)[4],
                                           float (&pw)[4]) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int idx = threadIdx.x + t * 256;
        const int r = idx / BK, kk = idx % BK;
        const int64_t gr = row0 + r;
        const int gk = k0 + kk;
        float v = 0.f;
        if (gr < g.m && gk < g.k) {
            v = g.a[gr * g.lda + gk];
            if (g.a_pre) v *= silu_grad(g.a_pre[gr * g.lda_pre + gk]);
        }
        pa[t] = v;
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int idx = threadIdx.x + t * 256;
        float v = 0.f;
        if (g.trans_w) {
            const int c = idx / BK, kk = idx % BK;
            const int gc = col0 + c, gk = k0 + kk;
            if (gc < g.n && gk < g.k) v = g.w[int64_t(gc) * g.ldw + gk];
        } else {
            const int kk = idx / BN, c = idx % BN;
            const int gc = col0 + c, gk = k0 + kk;
            if (gc < g.n && gk < g.k) v = g.w[int64_t(gk) * g.ldw + gc];
        }
        pw[t] = v;
    }
}

__device__ __forceinline__ void store_slice(const GemmArgs& g, float (*As)[BM + 4], float (*Ws)[BN + 4],
                                            const float (&pa)[4], const float (&pw)[4]) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int idx = threadIdx.x + t * 256;
        As[idx % BK][idx / BK] = pa[t];
        if (g.trans_w) Ws[idx % BK][idx / BK] = pw[t];
        else Ws[idx / BN][idx % BN] = pw[t];
    }
}

// K slices double-buffered: the next slice's global loads are in flight (registers) while the current
// slice's products run from shared memory; one barrier per slice
__global__ void __launch_bounds__(256) sgemm_kernel(GemmArgs g) {
    __shared__ float As[2][BK][BM + 4];
    __shared__ float Ws[2][BK][BN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int64_t row0 = int64_t(blockIdx.x) * BM;
    const int col0 = blockIdx.y * BN;
    float acc[4][4] = {};
    float pa[4], pw[4];
    load_slice(g, row0, col0, 0, pa, pw);
    store_slice(g, As[0], Ws[0], pa, pw);
    __syncthreads();
    const int slices = (g.k + BK - 1) / BK;
    for (int sl = 0; sl < slices; ++sl) {
        const int buf = sl & 1;
        if (sl + 1 < slices) load_slice(g, row0, col0, (sl + 1) * BK, pa, pw);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[buf][kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = Ws[buf][kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        // the other buffer was last read before the previous barrier
        if (sl + 1 < slices) store_slice(g, As[buf ^ 1], Ws[buf ^ 1], pa, pw);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gr = row0 + ty + 16 * i;
        if (gr >= g.m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gc = col0 + tx + 16 * j;
            if (gc >= g.n) continue;
            float v = acc[i][j];
            if (g.bias) v += g.bias[gc];
            if (g.y_pre) g.y_pre[gr * g.ldy_pre + gc] = v;
            if (g.act == 1) v = silu(v);
            float* dst = g.y + gr * g.ldy + gc;
            *dst = g.accumulate ? *dst + v : v;
        }
    }
}

}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_gemm_f32(const float* a, int64_t lda, const float* a_pre, int64_t lda_pre, const float* w,
                        int64_t ldw, int32_t trans_w, const float* bias, float* y, int64_t ldy, float* y_pre,
                        int64_t ldy_pre, int64_t m, int32_t n, int32_t k, int32_t act, int32_t accumulate,
                        void* stream) {
    if (a == nullptr || w == nullptr || y == nullptr || m < 0 || n < 0 || k < 0 || act < 0 || act > 1 ||
        lda < k || ldy < n || (trans_w ? ldw < k : ldw < n) || (a_pre != nullptr && lda_pre < k) ||
        (y_pre != nullptr && ldy_pre < n))
        return FMD_ERR_INVALID_ARGUMENT;
    if (m == 0 || n == 0) return FMD_OK;
    if ((m + BM - 1) / BM > 0x7fffffff || (n + BN - 1) / BN > 65535) return FMD_ERR_UNSUPPORTED;
    GemmArgs g{a, lda, a_pre, lda_pre, w, ldw, trans_w, bias, y, ldy, y_pre, ldy_pre, m, n, k, act, accumulate};
    const dim3 grid(unsigned((m + BM - 1) / BM), (n + BN - 1) / BN);
    sgemm_kernel<<<grid, 256, 0, as_stream(stream)>>>(g);
    return check_launch();
}

}  // extern "C"
