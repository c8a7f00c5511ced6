// The MACE-architecture step in a few fused kernels (the whole-step path).
//
// A 135-atom step is latency-bound: the unfused model launches ~60 small
// kernels. Here one step of an L-layer model is
//   edge_fwd        geometry + radial basis + the radial MLP of every layer
//                   (32-edge tiles, hidden activations in shared memory)
//   message(l)      gather -> tensor-product message -> receiver segment sum
//                   (one CTA per receiver, warps over its edges, fixed-order
//                   combine: deterministic, no atomics)
//   node_fwd(l)     per group of same-element atoms: channel mixing, the
//                   symmetric contraction, the output mixing, the skip
//                   connection, the readout and the next layer's up-mixing
//   node_last       the last layer's node update, its readout, the node
//                   energies, and the start of the backward (to dA)
//   msg_bwd_edge(l) per receiver run: dR and dY (warp per edge)
//   sender_node(l)  per sender run: the gathered rows' gradient, the
//                   up-mixing backward and the previous layer's node backward
//   edge_bwd        the radial MLP backward (recomputed forward) of every
//                   layer and the geometry backward: dE/dr_e per edge
//   forces          F_a = sum over received edges - sum over sent edges of
//                   dE/dr_e (both CSRs), the per-system energy sums
// From the tensor-core threshold on (the large replica unions), edge_fwd and
// edge_bwd are replaced by a geometry kernel, the radial MLPs as chained
// tcgen05 3xTF32 GEMMs on the pre-activations (fmd_gemm_tf32x3 with the SiLU
// on its input operand, and the SiLU-derivative gate in the backward), and a
// geometry backward kernel.
// Weights are frozen; the host prepares transposed copies once so every
// channel-mixing loop reads weights coalesced (thread = output channel).

#include "common.cuh"

namespace fmd {

constexpr int kMaxLayers = 4;
constexpr int kH = 64;        // radial MLP width
constexpr int kTF = 16;       // edges per tile of the forward edge kernel
constexpr int kMaxPC = 512;   // P*C of a layer's radial output (C <= 128)
constexpr int kTB = 16;       // edges per tile of the backward edge kernel
constexpr int kG = 4;         // atoms per group of the node kernels
constexpr float kS3 = 1.7320508075688772f;
constexpr float kIS3 = 0.5773502691896258f;

struct FusedWeights {
    // radial MLP per layer: transposed [in][out] for the forward, original [out][in] for the backward
    const float* w1t[kMaxLayers];
    const float* w2t[kMaxLayers];
    const float* w3t[kMaxLayers];
    const float* w4t[kMaxLayers];
    const float* w1[kMaxLayers];
    const float* w2[kMaxLayers];
    const float* w3[kMaxLayers];
    const float* w4[kMaxLayers];
    // channel mixing: original [out][in] and transposed [in][out]
    const float* lin0[kMaxLayers];
    const float* lin1[kMaxLayers];
    const float* lin0t[kMaxLayers];
    const float* lin1t[kMaxLayers];
    const float* out0[kMaxLayers];
    const float* out1[kMaxLayers];
    const float* out0t[kMaxLayers];
    const float* out1t[kMaxLayers];
    const float* up0[kMaxLayers];
    const float* up1[kMaxLayers];
    const float* up0t[kMaxLayers];
    const float* up1t[kMaxLayers];
    const float* prod0[kMaxLayers];   // [Z][5][C]
    const float* prod1[kMaxLayers];   // [Z][4][C]
    const float* skip0[kMaxLayers];   // [Z][in][out]
    const float* skip1[kMaxLayers];
    const float* skip0t[kMaxLayers];  // [Z][out][in]
    const float* skip1t[kMaxLayers];
    const float* s_t0;                // [Z][C]: layer 0's up-mixing of the embedding
    const float* r0;                  // [C] readout of layer 0
    const float* ra;                  // [RH][C]
    const float* rb;                  // [RH]
    const double* e0;                 // [Z]
    double scale, shift;
    int n_layers, n_basis, poly_p, readout_hidden;
    float r_max, inv_avg;
    // tensor-core radial MLP: TF32 splits of W2, W3, W4 as [out][in] and as [in][out]
    const float* tc_hi[3][kMaxLayers];
    const float* tc_lo[3][kMaxLayers];
    const float* tc_t_hi[3][kMaxLayers];
    const float* tc_t_lo[3][kMaxLayers];
    int64_t tc_min_edges;             // 0: never
    // the node path's channel mixings on the tensor cores: TF32 splits of lin0, lin1, out0, out1, up0,
    // up1 as [out][in] (m = 0..5, the forward mixings) and as [in][out] (m = 6..11, their backward)
    const float* ntc_hi[12][kMaxLayers];
    const float* ntc_lo[12][kMaxLayers];
    // and the per-element skip mixings: splits of skip0t (0, the forward) and skip0 (1, the backward)
    const float* skip_hi[2][kMaxLayers];
    const float* skip_lo[2][kMaxLayers];
};

// per-layer activations
struct FusedState {
    float* R[kMaxLayers];       // [E][P*C]
    float* dR[kMaxLayers];
    float* s_t[kMaxLayers];     // [N][C] (layer 0: unused, the table)
    float* v_t[kMaxLayers];     // [N][3][C]
    float* A0[kMaxLayers];      // [N][C] aggregated messages
    float* A1[kMaxLayers];      // [N][3][C]
    float* A0l[kMaxLayers];     // after the channel mixing
    float* A1l[kMaxLayers];
    float* s_out[kMaxLayers];   // layer outputs
    float* v_out[kMaxLayers];
    float* dA0[kMaxLayers];
    float* dA1[kMaxLayers];
    float* ds_skip[kMaxLayers]; // gradient of layer l's input from its skip connection
    float* dv_skip[kMaxLayers];
    float4* ysh;                // [E] (sqrt3 u, d)
    float* dY;                  // [E][3]
    float* g_r;                 // [E][3] dE/dr_e
    float* e_term0;             // [N]
    double* node_energy;        // [N]
    const int32_t* elem;        // [N]
    const int32_t* groups;      // [n_groups][kG] atom ids (-1 padding), same element per group
    int64_t n_groups;
    float* pre[3][kMaxLayers];  // [E][kH] radial pre-activations p1..p3 (tensor-core path; gradients in place)
    int32_t* flags;
    const int32_t* elem_order;  // [N] atoms sorted by element (the tensor-core skip mixings)
    const int32_t* elem_rank;   // [N] its inverse
    int64_t n_runs;             // element runs (element, first, count) over elem_order, on the host
    const int64_t* runs_host;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_g(float x) {
    const float s = 1.0f / (1.0f + expf(-x));
    return s * (1.0f + x * (1.0f - s));
}

__device__ __forceinline__ void cutoff_poly(float d, float r_max, int pp, float& f, float& df) {
    const float x = d / r_max;
    if (!(x < 1.0f)) {
        f = 0.f;
        df = 0.f;
        return;
    }
    const float p = float(pp);
    const float a = (p + 1.f) * (p + 2.f) * 0.5f, b = p * (p + 2.f), c = p * (p + 1.f) * 0.5f;
    const float xpm1 = powf(x, p - 1.f);
    const float xp = xpm1 * x;
    f = 1.f - a * xp + b * xp * x - c * xp * x * x;
    df = (-a * p * xpm1 + b * (p + 1.f) * xp - c * (p + 2.f) * xp * x) / r_max;
}

// ---------------------------------------------------------------- edge forward

struct EdgeArgs {
    const float* pos;
    const float* cell;
    const int32_t* edge_index;
    const float* edge_image;
    int64_t n_edges;           // rows of the edge arrays
    const int64_t* n_real;     // device count of the real rows (padding rows are skipped), or null
    int C;
};

constexpr int kHS = kH + 4;   // row stride of activation tiles (16-byte rows, broadcast float4 reads)
constexpr int kWS = kH + 1;   // row stride of staged weights (conflict-free row and column walks)

struct EdgeFwdSmem {
    float phi[kTF][16];
    float h[2][kTF][kHS];
    float w1[16][kH];          // W1^T [basis][hidden]
    float w2[kH][kWS];         // W2^T [in][out]
    float w3[kH][kWS];
};

// stage one layer's radial weights W1^T, W2^T, W3^T in shared memory (float4 loads, unrolled; NT threads)
template <int NT = 256>
__device__ __forceinline__ void stage_radial(float (*w1)[kH], float (*w2)[kWS], float (*w3)[kWS],
                                             const FusedWeights& w, int L) {
    const float4* g2 = reinterpret_cast<const float4*>(w.w2t[L]);
    const float4* g3 = reinterpret_cast<const float4*>(w.w3t[L]);
#pragma unroll
    for (int r = 0; r < kH * kH / 4 / NT; ++r) {
        const int idx = threadIdx.x + NT * r;  // float4 index
        const float4 a = g2[idx], b = g3[idx];
        const int row = (idx * 4) / kH, col = (idx * 4) % kH;
        w2[row][col] = a.x; w2[row][col + 1] = a.y; w2[row][col + 2] = a.z; w2[row][col + 3] = a.w;
        w3[row][col] = b.x; w3[row][col + 1] = b.y; w3[row][col + 2] = b.z; w3[row][col + 3] = b.w;
    }
    for (int idx = threadIdx.x; idx < w.n_basis * kH; idx += NT) w1[idx / kH][idx % kH] = w.w1t[L][idx];
}

// out[e][k] = act(sum_c in[e][c] W[c][k]) for the tile (thread k = t % 64, NT / 64 edge groups)
template <int TE, bool ACT, int NT = 256>
__device__ __forceinline__ void hidden_layer(const float (*in)[kHS], const float (*W)[kWS], float (*out)[kHS],
                                             float (*pre)[kHS]) {
    constexpr int EPG = TE / (NT / kH);
    const int k = threadIdx.x % kH, eg = threadIdx.x / kH;
    float acc[EPG];
#pragma unroll
    for (int m = 0; m < EPG; ++m) acc[m] = 0.f;
#pragma unroll 4
    for (int c = 0; c < kH; c += 4) {
        const float w0 = W[c][k], w1 = W[c + 1][k], w2 = W[c + 2][k], w3 = W[c + 3][k];
#pragma unroll
        for (int m = 0; m < EPG; ++m) {
            const float4 x = *reinterpret_cast<const float4*>(&in[eg * EPG + m][c]);
            acc[m] = fmaf(x.x, w0, acc[m]);
            acc[m] = fmaf(x.y, w1, acc[m]);
            acc[m] = fmaf(x.z, w2, acc[m]);
            acc[m] = fmaf(x.w, w3, acc[m]);
        }
    }
#pragma unroll
    for (int m = 0; m < EPG; ++m) {
        if (pre) pre[eg * EPG + m][k] = acc[m];
        out[eg * EPG + m][k] = ACT ? silu_f(acc[m]) : acc[m];
    }
}

__device__ __forceinline__ int64_t real_edges(const EdgeArgs& a) {
    const int64_t n = a.n_real ? *a.n_real : a.n_edges;
    return n < a.n_edges ? n : a.n_edges;
}

// R[e][n] = sum_c h3[e][c] W4^T[c][n] for one tile, PC columns (thread columns t, t+256, ...), W4^T
// staged in shared memory
template <int PC>
__device__ __forceinline__ void radial_out(const float (*h)[kHS], const float* w4s, float* __restrict__ R, int64_t e0,
                                           int ne) {
#pragma unroll
    for (int n = threadIdx.x; n < PC; n += 256) {
        float acc[kTF];
#pragma unroll
        for (int e = 0; e < kTF; ++e) acc[e] = 0.f;
#pragma unroll 4
        for (int c = 0; c < kH; c += 4) {
            const float w0 = w4s[(c + 0) * PC + n], w1 = w4s[(c + 1) * PC + n];
            const float w2 = w4s[(c + 2) * PC + n], w3 = w4s[(c + 3) * PC + n];
#pragma unroll
            for (int e = 0; e < kTF; ++e) {
                const float4 x = *reinterpret_cast<const float4*>(&h[e][c]);
                acc[e] = fmaf(x.x, w0, fmaf(x.y, w1, fmaf(x.z, w2, fmaf(x.w, w3, acc[e]))));
            }
        }
#pragma unroll
        for (int e = 0; e < kTF; ++e)
            if (e < ne) R[(e0 + e) * PC + n] = acc[e];
    }
}

// stage W4^T [kH][PC] of one layer in shared memory (float4 loads issued together)
template <int PC>
__device__ __forceinline__ void stage_w4(float* w4s, const float* __restrict__ w4t) {
    const float4* src = reinterpret_cast<const float4*>(w4t);
    float4* dst = reinterpret_cast<float4*>(w4s);
#pragma unroll 8
    for (int idx = threadIdx.x; idx < kH * PC / 4; idx += 256) dst[idx] = src[idx];
}

// geometry, radial features and the radial MLP of every layer for one 16-edge tile (the output
// weights W4^T of the layer staged in shared memory after the struct: kH x 4C floats)
template <int C>
__global__ void __launch_bounds__(256) edge_fwd_kernel(EdgeArgs a, FusedWeights w, FusedState st) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    EdgeFwdSmem& m = *reinterpret_cast<EdgeFwdSmem*>(smem_raw);
    float* w4s = reinterpret_cast<float*>(smem_raw + sizeof(EdgeFwdSmem));
    const int t = threadIdx.x;
    const float pref = sqrtf(2.0f / w.r_max);
    const int64_t n_edges = real_edges(a);
    const int64_t n_tiles = (n_edges + kTF - 1) / kTF;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t e0 = tile * kTF;
        const int ne = int(n_edges - e0 < kTF ? n_edges - e0 : kTF);
        __syncthreads();
        if (t < kTF) {
            const int64_t e = e0 + t;
            float d = 0.f;
            if (t < ne) {
                const int64_t i = a.edge_index[2 * e], j = a.edge_index[2 * e + 1];
                const float ix = a.edge_image[3 * e], iy = a.edge_image[3 * e + 1], iz = a.edge_image[3 * e + 2];
                const float* c = a.cell;
                const float rx = (a.pos[3 * j] - a.pos[3 * i]) + ((ix * c[0] + iy * c[3]) + iz * c[6]);
                const float ry = (a.pos[3 * j + 1] - a.pos[3 * i + 1]) + ((ix * c[1] + iy * c[4]) + iz * c[7]);
                const float rz = (a.pos[3 * j + 2] - a.pos[3 * i + 2]) + ((ix * c[2] + iy * c[5]) + iz * c[8]);
                d = sqrtf((rx * rx + ry * ry) + rz * rz);
                const float inv = d > 0.f ? 1.0f / d : 0.f;
                st.ysh[e] = make_float4(kS3 * rx * inv, kS3 * ry * inv, kS3 * rz * inv, d);
            }
            float f, df;
            cutoff_poly(d, w.r_max, w.poly_p, f, df);
            const float inv = d > 0.f ? 1.0f / d : 0.f;
            for (int n = 0; n < w.n_basis; ++n) {
                const float k = float(n + 1) * 3.14159265358979323846f / w.r_max;
                m.phi[t][n] = d > 0.f ? pref * sinf(k * d) * inv * f : 0.f;
            }
        }
        for (int L = 0; L < w.n_layers; ++L) {
            __syncthreads();
            stage_radial(m.w1, m.w2, m.w3, w, L);
            if (L == 0) stage_w4<2 * C>(w4s, w.w4t[L]);
            else stage_w4<4 * C>(w4s, w.w4t[L]);
            __syncthreads();
            for (int idx = t; idx < kTF * kH; idx += 256) {
                const int e = idx / kH, k = idx % kH;
                float acc = 0.f;
                for (int n = 0; n < w.n_basis; ++n) acc = fmaf(m.phi[e][n], m.w1[n][k], acc);
                m.h[0][e][k] = silu_f(acc);
            }
            __syncthreads();
            hidden_layer<kTF, true>(m.h[0], m.w2, m.h[1], nullptr);
            __syncthreads();
            hidden_layer<kTF, true>(m.h[1], m.w3, m.h[0], nullptr);
            __syncthreads();
            if (L == 0) radial_out<2 * C>(m.h[0], w4s, st.R[L], e0, ne);
            else radial_out<4 * C>(m.h[0], w4s, st.R[L], e0, ne);
        }
    }
}

// ------------------------------------------------------------------ messages

// N consecutive floats of a lane (16-, 8- or 4-byte aligned rows): one vector access
template <int N>
__device__ __forceinline__ void ldv(const float* p, float (&v)[N]) {
    if constexpr (N == 4) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (N == 2) {
        const float2 x = *reinterpret_cast<const float2*>(p);
        v[0] = x.x; v[1] = x.y;
    } else {
#pragma unroll
        for (int q = 0; q < N; ++q) v[q] = p[q];
    }
}

template <int N>
__device__ __forceinline__ void stv(float* p, const float (&v)[N]) {
    if constexpr (N == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else if constexpr (N == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int q = 0; q < N; ++q) p[q] = v[q];
    }
}

struct GraphArgs {
    const int32_t* edge_index;
    const int64_t* recv_off;
    const int64_t* send_off;
    const int32_t* send_perm;
    int64_t n_atoms;
};

// A(l) of every receiver; kMsgWarps warps over the receiver's edges, fixed-order combine of the warp
// partials (a pairwise tree)
constexpr int kMsgWarps = 8;
template <int C, int P>
__global__ void __launch_bounds__(32 * kMsgWarps) message_fused_kernel(GraphArgs g, FusedWeights w, FusedState st,
                                                                      int L) {
    constexpr int CPL = C / 32;
    __shared__ float s_part[kMsgWarps][4][C];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* R = st.R[L];
    const float* v_t = st.v_t[L];
    for (int64_t i = blockIdx.x; i < g.n_atoms; i += gridDim.x) {
        float a0[CPL], ax[CPL], ay[CPL], az[CPL];
#pragma unroll
        for (int q = 0; q < CPL; ++q) a0[q] = ax[q] = ay[q] = az[q] = 0.f;
        const int64_t beg = g.recv_off[i], end = g.recv_off[i + 1];
        for (int64_t e = beg + warp; e < end; e += kMsgWarps) {
            const int64_t j = g.edge_index[2 * e + 1];
            const float4 y = st.ysh[e];
            const float* Re = R + e * (P * C) + lane * CPL;
            const float* srow = ((L == 0) ? w.s_t0 + int64_t(st.elem[j]) * C : st.s_t[L] + j * C) + lane * CPL;
            float sv[CPL], r0[CPL], r1[CPL], r2[CPL], r3[CPL], vx[CPL], vy[CPL], vz[CPL];
            ldv<CPL>(srow, sv);
            ldv<CPL>(Re, r0);
            ldv<CPL>(Re + C, r1);
            if constexpr (P == 4) {
                const float* vrow = v_t + j * 3 * C + lane * CPL;
                ldv<CPL>(Re + 2 * C, r2);
                ldv<CPL>(Re + 3 * C, r3);
                ldv<CPL>(vrow, vx);
                ldv<CPL>(vrow + C, vy);
                ldv<CPL>(vrow + 2 * C, vz);
            }
#pragma unroll
            for (int q = 0; q < CPL; ++q) {
                const float s = sv[q];
                a0[q] = fmaf(r0[q], s, a0[q]);
                const float m1 = r1[q] * s;
                ax[q] = fmaf(m1, y.x, ax[q]);
                ay[q] = fmaf(m1, y.y, ay[q]);
                az[q] = fmaf(m1, y.z, az[q]);
                if constexpr (P == 4) {
                    ax[q] = fmaf(r2[q], vx[q], ax[q]);
                    ay[q] = fmaf(r2[q], vy[q], ay[q]);
                    az[q] = fmaf(r2[q], vz[q], az[q]);
                    a0[q] = fmaf(r3[q] * kIS3, (vx[q] * y.x + vy[q] * y.y) + vz[q] * y.z, a0[q]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            const int k = lane * CPL + q;
            s_part[warp][0][k] = a0[q];
            s_part[warp][1][k] = ax[q];
            s_part[warp][2][k] = ay[q];
            s_part[warp][3][k] = az[q];
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < 4 * C; idx += 32 * kMsgWarps) {
            const int comp = idx / C, k = idx % C;
            float part[kMsgWarps];
#pragma unroll
            for (int wv = 0; wv < kMsgWarps; ++wv) part[wv] = s_part[wv][comp][k];
#pragma unroll
            for (int width = kMsgWarps / 2; width > 0; width /= 2)
#pragma unroll
                for (int wv = 0; wv < width; ++wv) part[wv] = part[wv] + part[wv + width];
            const float v = part[0] * w.inv_avg;
            if (comp == 0) st.A0[L][i * C + k] = v;
            else st.A1[L][i * 3 * C + (comp - 1) * C + k] = v;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------ node kernels
//
// A CTA of 4*C threads owns a group of G same-element atoms: G = kG = 4
// (the element groups of the host), or G = 1 (each entry of the group table
// on its own CTA, empty entries skipped) when there are fewer groups than SMs,
// so a small system fills the GPU with 4x the CTAs. Channel
// mixings [rows x C] . [C x C] split the reduction over c into 4 quarters
// (thread (k, q) = output channel k, quarter q): each thread issues its 32
// weight loads at once, so a matrix costs one L2 round trip; the quarters
// are combined in a fixed order in shared memory. Elementwise phases use
// thread (k, g) = channel k of atom g (g >= G: idle rows of the 4-atom
// shared-memory tiles, never written to global memory). The arithmetic of an
// atom's row does not depend on G: both forms give the same bits.

constexpr int kGV = kG * 3;
constexpr int kQ = 4;  // reduction quarters (== kG: the same threads serve both layouts)

template <int C>
struct NodeSmem {
    float s[kG][C];             // scalar rows of the group
    float v[kGV][C];            // vector rows (atom-major, component-minor)
    float t[kG][C];
    float tv[kGV][C];
    float red[kQ][kG + kGV][C]; // quarter partials
    float ra[32][C];            // readout weights (node_last)
    float pre[kG][32];
    float sc[kG][32];           // per-atom scalar reduction scratch
};

// outs[r][k] = sum_c xs[r][c] W0[c*C + k] (r < NS) and outv[r][k] = sum_c xv[r][c] W1[c*C + k]
// (r < NV); out may alias x. All 4*C threads call it; it ends with a barrier.
template <int C, int NS, int NV>
__device__ __forceinline__ void mix_rows(const float (*xs)[C], const float* __restrict__ W0, const float (*xv)[C],
                                         const float* __restrict__ W1, float (*outs)[C], float (*outv)[C],
                                         float (*red)[kG + kGV][C]) {
    constexpr int CQ = C / kQ;
    const int k = threadIdx.x % C, q = threadIdx.x / C;
    float acc[NS + NV];
#pragma unroll
    for (int r = 0; r < NS + NV; ++r) acc[r] = 0.f;
    // four input channels per step: one 16-byte shared-memory read of a row serves four FMAs (the row
    // operands, not the FMA pipe, bound a one-channel loop); every accumulator still adds c in order
    static_assert(CQ % 4 == 0, "a quarter of the channels must be a multiple of 4");
#pragma unroll 2
    for (int cc = 0; cc < CQ; cc += 4) {
        const int c = q * CQ + cc;
        if constexpr (NS > 0) {
            float w0[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) w0[j] = W0[(c + j) * C + k];
#pragma unroll
            for (int r = 0; r < NS; ++r) {
                const float4 x = *reinterpret_cast<const float4*>(&xs[r][c]);
                acc[r] = fmaf(x.x, w0[0], acc[r]);
                acc[r] = fmaf(x.y, w0[1], acc[r]);
                acc[r] = fmaf(x.z, w0[2], acc[r]);
                acc[r] = fmaf(x.w, w0[3], acc[r]);
            }
        }
        if constexpr (NV > 0) {
            float w1[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) w1[j] = W1[(c + j) * C + k];
#pragma unroll
            for (int r = 0; r < NV; ++r) {
                const float4 x = *reinterpret_cast<const float4*>(&xv[r][c]);
                acc[NS + r] = fmaf(x.x, w1[0], acc[NS + r]);
                acc[NS + r] = fmaf(x.y, w1[1], acc[NS + r]);
                acc[NS + r] = fmaf(x.z, w1[2], acc[NS + r]);
                acc[NS + r] = fmaf(x.w, w1[3], acc[NS + r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < NS + NV; ++r) red[q][r][k] = acc[r];
    __syncthreads();
    for (int idx = threadIdx.x; idx < (NS + NV) * C; idx += kQ * C) {
        const int r = idx / C, kk = idx % C;
        const float y = (red[0][r][kk] + red[1][r][kk]) + (red[2][r][kk] + red[3][r][kk]);
        if (r < NS) outs[r][kk] = y;
        else outv[r - NS][kk] = y;
    }
    __syncthreads();
}

// sum over the C channels of atom g (threads g*C .. g*C+C-1), result returned to every thread of atom g
template <int C>
__device__ __forceinline__ float atom_sum(float x, float (*sc)[32]) {
    const int g = threadIdx.x / C, k = threadIdx.x % C;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) x += __shfl_xor_sync(0xffffffffu, x, d);
    if ((k & 31) == 0) sc[g][k >> 5] = x;
    __syncthreads();
    float y = 0.f;
    for (int wv = 0; wv < C / 32; ++wv) y += sc[g][wv];
    __syncthreads();
    return y;
}

// the atoms of work unit grp: G consecutive entries of the group table, -1 past them
template <int G>
__device__ __forceinline__ void group_atoms(const FusedState& st, int64_t grp, int (&atoms)[kG]) {
#pragma unroll
    for (int g = 0; g < kG; ++g) atoms[g] = g < G ? st.groups[grp * G + g] : -1;
}

// work units of the node kernels: groups of 4, or single entries of the group table
template <int G>
__device__ __forceinline__ int64_t node_units(const FusedState& st) {
    return st.n_groups * (kG / G);
}

// forward node update of a non-last layer L
template <int C, int G>
__global__ void __launch_bounds__(kQ * C, 2) node_fwd_kernel(FusedWeights w, FusedState st, int L) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    NodeSmem<C>& m = *reinterpret_cast<NodeSmem<C>*>(smem_raw);
    const int k = threadIdx.x % C, g = threadIdx.x / C;
    for (int64_t grp = blockIdx.x; grp < node_units<G>(st); grp += gridDim.x) {
        int atoms[kG];
        group_atoms<G>(st, grp, atoms);
        if (atoms[0] < 0) continue;  // an empty entry of the table (uniform over the CTA)
        const int64_t z = st.elem[atoms[0]];
        const int my = atoms[g];
        const int64_t i = my < 0 ? atoms[0] : my;
        __syncthreads();
        m.s[g][k] = st.A0[L][i * C + k];
#pragma unroll
        for (int c = 0; c < 3; ++c) m.v[g * 3 + c][k] = st.A1[L][i * 3 * C + c * C + k];
        if (L > 0) {
            m.t[g][k] = st.s_out[L - 1][i * C + k];
#pragma unroll
            for (int c = 0; c < 3; ++c) m.tv[g * 3 + c][k] = st.v_out[L - 1][i * 3 * C + c * C + k];
        }
        __syncthreads();
        mix_rows<C, G, 3 * G>(m.s, w.lin0t[L], m.v, w.lin1t[L], m.s, m.v, m.red);
        if (L > 0) mix_rows<C, G, 3 * G>(m.t, w.skip0[L] + z * C * C, m.tv, w.skip1[L] + z * C * C, m.t, m.tv, m.red);
        // symmetric contraction (thread (k, g))
        const float aa = m.s[g][k];
        const float vx = m.v[g * 3][k], vy = m.v[g * 3 + 1][k], vz = m.v[g * 3 + 2][k];
        if (my >= 0) {
            st.A0l[L][my * int64_t(C) + k] = aa;
            st.A1l[L][my * int64_t(3 * C) + k] = vx;
            st.A1l[L][my * int64_t(3 * C) + C + k] = vy;
            st.A1l[L][my * int64_t(3 * C) + 2 * C + k] = vz;
        }
        const float* p0 = w.prod0[L] + z * 5 * C + k;
        const float* p1 = w.prod1[L] + z * 4 * C + k;
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float b0 = (((p0[0] * aa + p0[C] * aa * aa) + p0[2 * C] * q) + p0[3 * C] * aa * aa * aa) + p0[4 * C] * aa * q;
        const float cc = ((p1[0] + p1[C] * aa) + p1[2 * C] * aa * aa) + p1[3 * C] * q;
        __syncthreads();
        m.s[g][k] = b0;
        m.v[g * 3][k] = cc * vx;
        m.v[g * 3 + 1][k] = cc * vy;
        m.v[g * 3 + 2][k] = cc * vz;
        __syncthreads();
        mix_rows<C, G, 3 * G>(m.s, w.out0t[L], m.v, w.out1t[L], m.s, m.v, m.red);
        float so = m.s[g][k];
        float vo[3] = {m.v[g * 3][k], m.v[g * 3 + 1][k], m.v[g * 3 + 2][k]};
        if (L > 0) {
            so += m.t[g][k];
#pragma unroll
            for (int c = 0; c < 3; ++c) vo[c] += m.tv[g * 3 + c][k];
        }
        if (my >= 0) {
            st.s_out[L][my * int64_t(C) + k] = so;
#pragma unroll
            for (int c = 0; c < 3; ++c) st.v_out[L][my * int64_t(3 * C) + c * C + k] = vo[c];
        }
        if (L == 0) {  // readout of layer 0: e_term0 = s . r0
            const float e = atom_sum<C>(so * w.r0[k], m.sc);
            if (k == 0 && my >= 0) st.e_term0[my] = e;
        }
        __syncthreads();
        m.s[g][k] = so;
#pragma unroll
        for (int c = 0; c < 3; ++c) m.v[g * 3 + c][k] = vo[c];
        __syncthreads();
        // the next layer's up-mixing
        mix_rows<C, G, 3 * G>(m.s, w.up0t[L + 1], m.v, w.up1t[L + 1], m.s, m.v, m.red);
        if (my >= 0) {
            st.s_t[L + 1][my * int64_t(C) + k] = m.s[g][k];
#pragma unroll
            for (int c = 0; c < 3; ++c) st.v_t[L + 1][my * int64_t(3 * C) + c * C + k] = m.v[g * 3 + c][k];
        }
    }
}

// the last layer: node update, readout, node energies, and the backward to dA(L)
template <int C, int G>
__global__ void __launch_bounds__(kQ * C, 2) node_last_kernel(FusedWeights w, FusedState st, int L) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    NodeSmem<C>& m = *reinterpret_cast<NodeSmem<C>*>(smem_raw);
    const int k = threadIdx.x % C, g = threadIdx.x / C;
    const int RH = w.readout_hidden;
    for (int idx = threadIdx.x; idx < RH * C; idx += kQ * C) m.ra[idx / C][idx % C] = w.ra[idx];
    for (int64_t grp = blockIdx.x; grp < node_units<G>(st); grp += gridDim.x) {
        int atoms[kG];
        group_atoms<G>(st, grp, atoms);
        if (atoms[0] < 0) continue;  // an empty entry of the table (uniform over the CTA)
        const int64_t z = st.elem[atoms[0]];
        const int my = atoms[g];
        const int64_t i = my < 0 ? atoms[0] : my;
        __syncthreads();
        m.s[g][k] = st.A0[L][i * C + k];
#pragma unroll
        for (int c = 0; c < 3; ++c) m.v[g * 3 + c][k] = st.A1[L][i * 3 * C + c * C + k];
        m.t[g][k] = L > 0 ? st.s_out[L - 1][i * C + k] : 0.f;
        __syncthreads();
        mix_rows<C, G, 3 * G>(m.s, w.lin0t[L], m.v, w.lin1t[L], m.s, m.v, m.red);
        if (L > 0) mix_rows<C, G, 0>(m.t, w.skip0[L] + z * C * C, nullptr, nullptr, m.t, nullptr, m.red);
        const float aa = m.s[g][k];
        const float vx = m.v[g * 3][k], vy = m.v[g * 3 + 1][k], vz = m.v[g * 3 + 2][k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float* p0 = w.prod0[L] + z * 5 * C + k;
        const float b0 = (((p0[0] * aa + p0[C] * aa * aa) + p0[2 * C] * q) + p0[3 * C] * aa * aa * aa) + p0[4 * C] * aa * q;
        __syncthreads();
        m.s[g][k] = b0;
        __syncthreads();
        mix_rows<C, G, 0>(m.s, w.out0t[L], nullptr, nullptr, m.s, nullptr, m.red);
        const float so = m.s[g][k] + (L > 0 ? m.t[g][k] : 0.f);
        float e0_term = 0.f;
        if (L == 0) e0_term = atom_sum<C>(so * w.r0[k], m.sc);  // a one-layer model: readout 0 as well
        __syncthreads();
        m.s[g][k] = so;
        __syncthreads();
        // readout MLP: pre_j = s . ra_j
        for (int idx = threadIdx.x; idx < G * RH; idx += kQ * C) {
            const int gg = idx / RH, j = idx % RH;
            float acc = 0.f;
            for (int c = 0; c < C; ++c) acc = fmaf(m.s[gg][c], m.ra[j][c], acc);
            m.pre[gg][j] = acc;
        }
        __syncthreads();
        if (k == 0 && my >= 0) {
            float e1 = 0.f;
            for (int j = 0; j < RH; ++j) e1 = fmaf(w.rb[j], silu_f(m.pre[g][j]), e1);
            const float et = L > 0 ? st.e_term0[my] : e0_term;
            st.node_energy[my] = w.e0[z] + w.scale * (double(et) + double(e1)) + w.shift;
        }
        // ---- backward: ds = scale * sum_j rb[j] silu'(pre_j) ra[j] (+ scale * r0 for a one-layer model)
        const float sc = float(w.scale);
        float acc = 0.f;
        for (int j = 0; j < RH; ++j) acc = fmaf(w.rb[j] * silu_g(m.pre[g][j]), m.ra[j][k], acc);
        float ds = sc * acc;
        if (L == 0) ds = fmaf(sc, w.r0[k], ds);
        __syncthreads();
        m.t[g][k] = ds;
        __syncthreads();
        if (L > 0) {
            mix_rows<C, G, 0>(m.t, w.skip0t[L] + z * C * C, nullptr, nullptr, m.v, nullptr, m.red);
            if (my >= 0) st.ds_skip[L][my * int64_t(C) + k] = m.v[g][k];
        }
        mix_rows<C, G, 0>(m.t, w.out0[L], nullptr, nullptr, m.t, nullptr, m.red);
        const float db0 = m.t[g][k];
        const float gq = db0 * (p0[2 * C] + p0[4 * C] * aa);
        const float da = db0 * (((p0[0] + 2.f * p0[C] * aa) + 3.f * p0[3 * C] * aa * aa) + p0[4 * C] * q);
        __syncthreads();
        m.s[g][k] = da;
        m.v[g * 3][k] = 2.f * gq * vx;
        m.v[g * 3 + 1][k] = 2.f * gq * vy;
        m.v[g * 3 + 2][k] = 2.f * gq * vz;
        __syncthreads();
        mix_rows<C, G, 3 * G>(m.s, w.lin0[L], m.v, w.lin1[L], m.s, m.v, m.red);
        if (my >= 0) {
            st.dA0[L][my * int64_t(C) + k] = m.s[g][k];
#pragma unroll
            for (int c = 0; c < 3; ++c) st.dA1[L][my * int64_t(3 * C) + c * C + k] = m.v[g * 3 + c][k];
        }
    }
}

// per receiver run: dR(l) and dY (warp per edge, lane channels; dY accumulated over layers); every
// output is one edge's, so the warps of a receiver give the same bits in any number or order
constexpr int kMsgBwdWarps = 8;

// one warp: U edges e0, e0 + stride, ... (those below end) of receiver gradient rows g0, gx, gy, gz,
// their loads issued together
template <int C, int P, int U>
__device__ __forceinline__ void msg_bwd_edges(const GraphArgs& g, const FusedWeights& w, const FusedState& st, int L,
                                              int accumulate_dy, const float* g0, const float* gx, const float* gy,
                                              const float* gz, int64_t e0, int64_t stride, int64_t end, int lane) {
    constexpr int CPL = C / 32;
    const float* R = st.R[L];
    float* dR = st.dR[L];
    int64_t ee[U];
    bool valid[U];
    float4 y[U];
    float sv[U][CPL], r1[U][CPL], r3[U][CPL], vx[U][CPL], vy[U][CPL], vz[U][CPL];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        valid[u] = e0 + u * stride < end;
        ee[u] = valid[u] ? e0 + u * stride : e0;
        const int64_t j = g.edge_index[2 * ee[u] + 1];
        y[u] = st.ysh[ee[u]];
        const float* Re = R + ee[u] * (P * C) + lane * CPL;
        const float* srow = ((L == 0) ? w.s_t0 + int64_t(st.elem[j]) * C : st.s_t[L] + j * C) + lane * CPL;
        ldv<CPL>(srow, sv[u]);
        ldv<CPL>(Re + C, r1[u]);
        if constexpr (P == 4) {
            const float* vrow = st.v_t[L] + j * 3 * C + lane * CPL;
            ldv<CPL>(Re + 3 * C, r3[u]);
            ldv<CPL>(vrow, vx[u]);
            ldv<CPL>(vrow + C, vy[u]);
            ldv<CPL>(vrow + 2 * C, vz[u]);
        }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
        if (!valid[u]) continue;
        const int64_t e = ee[u];
        float* dRe = dR + e * (P * C) + lane * CPL;
        float o0[CPL], o1[CPL], o2[CPL], o3[CPL];
        float px = 0.f, py = 0.f, pz = 0.f;
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            const float s = sv[u][q];
            const float gdy = (gx[q] * y[u].x + gy[q] * y[u].y) + gz[q] * y[u].z;
            o0[q] = g0[q] * s;
            o1[q] = s * gdy;
            const float c1 = r1[u][q] * s;
            px = fmaf(c1, gx[q], px);
            py = fmaf(c1, gy[q], py);
            pz = fmaf(c1, gz[q], pz);
            if constexpr (P == 4) {
                o2[q] = (gx[q] * vx[u][q] + gy[q] * vy[u][q]) + gz[q] * vz[u][q];
                o3[q] = g0[q] * ((vx[u][q] * y[u].x + vy[u][q] * y[u].y) + vz[u][q] * y[u].z) * kIS3;
                const float c3 = r3[u][q] * g0[q] * kIS3;
                px = fmaf(c3, vx[u][q], px);
                py = fmaf(c3, vy[u][q], py);
                pz = fmaf(c3, vz[u][q], pz);
            }
        }
        stv<CPL>(dRe, o0);
        stv<CPL>(dRe + C, o1);
        if constexpr (P == 4) {
            stv<CPL>(dRe + 2 * C, o2);
            stv<CPL>(dRe + 3 * C, o3);
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            px += __shfl_xor_sync(0xffffffffu, px, d);
            py += __shfl_xor_sync(0xffffffffu, py, d);
            pz += __shfl_xor_sync(0xffffffffu, pz, d);
        }
        if (lane == 0) {
            float* out = st.dY + 3 * e;
            if (accumulate_dy) {
                out[0] += px;
                out[1] += py;
                out[2] += pz;
            } else {
                out[0] = px;
                out[1] = py;
                out[2] = pz;
            }
        }
    }
}

// per_warp: each warp owns whole receiver runs (grid-stride over warps), two edges in flight; else a
// CTA per receiver with its warps over the run (few atoms: every SM busy)
template <int C, int P>
__global__ void __launch_bounds__(32 * kMsgBwdWarps) msg_bwd_edge_kernel(GraphArgs g, FusedWeights w, FusedState st,
                                                                        int L, int accumulate_dy, int per_warp) {
    constexpr int CPL = C / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t first = per_warp ? int64_t(blockIdx.x) * kMsgBwdWarps + warp : blockIdx.x;
    const int64_t step = per_warp ? int64_t(gridDim.x) * kMsgBwdWarps : gridDim.x;
    for (int64_t i = first; i < g.n_atoms; i += step) {
        float g0[CPL], gx[CPL], gy[CPL], gz[CPL];
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            const int k = lane * CPL + q;
            g0[q] = st.dA0[L][i * C + k] * w.inv_avg;
            gx[q] = st.dA1[L][i * 3 * C + k] * w.inv_avg;
            gy[q] = st.dA1[L][i * 3 * C + C + k] * w.inv_avg;
            gz[q] = st.dA1[L][i * 3 * C + 2 * C + k] * w.inv_avg;
        }
        const int64_t beg = g.recv_off[i], end = g.recv_off[i + 1];
        if (per_warp) {
            for (int64_t e = beg; e < end; e += 2)
                msg_bwd_edges<C, P, 2>(g, w, st, L, accumulate_dy, g0, gx, gy, gz, e, 1, end, lane);
        } else {
            for (int64_t e = beg + warp; e < end; e += kMsgBwdWarps)
                msg_bwd_edges<C, P, 1>(g, w, st, L, accumulate_dy, g0, gx, gy, gz, e, kMsgBwdWarps, end, lane);
        }
    }
}

// per sender: the gathered rows' gradient of layer L (ds_t, dv_t), the up-mixing backward into
// layer L-1's outputs, and layer L-1's node backward (to dA(L-1)). One atom group per CTA; the
// C threads of atom g reduce its sender run (warps over edges).
template <int C, int G>
__global__ void __launch_bounds__(kQ * C, 2) sender_node_kernel(GraphArgs gr, FusedWeights w, FusedState st, int L) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    NodeSmem<C>& m = *reinterpret_cast<NodeSmem<C>*>(smem_raw);
    // the C / 32 warps of atom g reduce its sender run (the same order whatever G: the results do not
    // depend on the grouping); with G < kG the warps of the idle atom slots skip it
    constexpr int CPL = C / 32, NW = C / 32;
    const int k = threadIdx.x % C, g = threadIdx.x / C;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ga = warp / NW, wa = warp % NW;  // ga == g
    float (*redf)[C] = reinterpret_cast<float (*)[C]>(&m.red[0][0][0]);  // [4 * warps][C] partials
    const int P = 4;
    const float* R = st.R[L];
    const int Lp = L - 1;
    for (int64_t grp = blockIdx.x; grp < node_units<G>(st); grp += gridDim.x) {
        int atoms[kG];
        group_atoms<G>(st, grp, atoms);
        if (atoms[0] < 0) continue;  // an empty entry of the table (uniform over the CTA)
        const int64_t z = st.elem[atoms[0]];
        const int my = atoms[g];
        const int64_t j = my < 0 ? atoms[0] : my;
        const int mw = atoms[ga];
        const int64_t jw = mw < 0 ? atoms[0] : mw;
        float ds[CPL], dx[CPL], dy[CPL], dz[CPL];
#pragma unroll
        for (int qq = 0; qq < CPL; ++qq) ds[qq] = dx[qq] = dy[qq] = dz[qq] = 0.f;
        for (int64_t t = gr.send_off[jw] + wa; ga < G && t < gr.send_off[jw + 1]; t += NW) {
            const int64_t e = gr.send_perm[t];
            const int64_t i = gr.edge_index[2 * e];
            const float4 y = st.ysh[e];
            const float* Re = R + e * (P * C) + lane * CPL;
            const float* a0 = st.dA0[L] + i * C + lane * CPL;
            const float* a1 = st.dA1[L] + i * 3 * C + lane * CPL;
            float r0[CPL], r1[CPL], r2v[CPL], r3v[CPL], d0[CPL], dxv[CPL], dyv[CPL], dzv[CPL];
            ldv<CPL>(Re, r0);
            ldv<CPL>(Re + C, r1);
            ldv<CPL>(Re + 2 * C, r2v);
            ldv<CPL>(Re + 3 * C, r3v);
            ldv<CPL>(a0, d0);
            ldv<CPL>(a1, dxv);
            ldv<CPL>(a1 + C, dyv);
            ldv<CPL>(a1 + 2 * C, dzv);
#pragma unroll
            for (int qq = 0; qq < CPL; ++qq) {
                const float g0 = d0[qq] * w.inv_avg;
                const float gx = dxv[qq] * w.inv_avg;
                const float gy = dyv[qq] * w.inv_avg;
                const float gz = dzv[qq] * w.inv_avg;
                ds[qq] = fmaf(r0[qq], g0, ds[qq]);
                ds[qq] = fmaf(r1[qq], (gx * y.x + gy * y.y) + gz * y.z, ds[qq]);
                const float r2 = r2v[qq], r3 = r3v[qq] * g0 * kIS3;
                dx[qq] = fmaf(r2, gx, fmaf(r3, y.x, dx[qq]));
                dy[qq] = fmaf(r2, gy, fmaf(r3, y.y, dy[qq]));
                dz[qq] = fmaf(r2, gz, fmaf(r3, y.z, dz[qq]));
            }
        }
        __syncthreads();
        // warp partials of atom ga -> rows (ga * NW + wa) * 4 + (s, x, y, z) of the partial block
#pragma unroll
        for (int qq = 0; qq < CPL; ++qq) {
            const int kk = lane * CPL + qq;
            redf[(ga * NW + wa) * 4 + 0][kk] = ds[qq];
            redf[(ga * NW + wa) * 4 + 1][kk] = dx[qq];
            redf[(ga * NW + wa) * 4 + 2][kk] = dy[qq];
            redf[(ga * NW + wa) * 4 + 3][kk] = dz[qq];
        }
        __syncthreads();
        {
            float sum[4] = {0.f, 0.f, 0.f, 0.f};
            if (g < G)
                for (int wv = 0; wv < NW; ++wv)
#pragma unroll
                    for (int c = 0; c < 4; ++c) sum[c] += redf[(g * NW + wv) * 4 + c][k];
            m.s[g][k] = sum[0];
#pragma unroll
            for (int c = 0; c < 3; ++c) m.v[g * 3 + c][k] = sum[1 + c];
        }
        __syncthreads();
        // up-mixing backward into layer Lp's outputs, plus the skip and readout parts
        mix_rows<C, G, 3 * G>(m.s, w.up0[L], m.v, w.up1[L], m.s, m.v, m.red);
        float dsi = m.s[g][k];
        float dvi[3] = {m.v[g * 3][k], m.v[g * 3 + 1][k], m.v[g * 3 + 2][k]};
        if (st.ds_skip[L]) dsi += st.ds_skip[L][j * C + k];
        if (st.dv_skip[L])
#pragma unroll
            for (int c = 0; c < 3; ++c) dvi[c] += st.dv_skip[L][j * 3 * C + c * C + k];
        if (Lp == 0) dsi = fmaf(float(w.scale), w.r0[k], dsi);  // layer 0 feeds the linear readout
        __syncthreads();
        m.t[g][k] = dsi;
#pragma unroll
        for (int c = 0; c < 3; ++c) m.tv[g * 3 + c][k] = dvi[c];
        __syncthreads();
        // layer Lp: out-mixing backward (into s/v) and skip backward (t/tv in place)
        mix_rows<C, G, 3 * G>(m.t, w.out0[Lp], m.tv, w.out1[Lp], m.s, m.v, m.red);
        if (Lp > 0) {
            mix_rows<C, G, 3 * G>(m.t, w.skip0t[Lp] + z * C * C, m.tv, w.skip1t[Lp] + z * C * C, m.t, m.tv, m.red);
            if (my >= 0) {
                st.ds_skip[Lp][my * int64_t(C) + k] = m.t[g][k];
#pragma unroll
                for (int c = 0; c < 3; ++c) st.dv_skip[Lp][my * int64_t(3 * C) + c * C + k] = m.tv[g * 3 + c][k];
            }
        }
        // product backward
        const float* p0 = w.prod0[Lp] + z * 5 * C + k;
        const float* p1 = w.prod1[Lp] + z * 4 * C + k;
        const float aa = st.A0l[Lp][j * C + k];
        const float vx = st.A1l[Lp][j * 3 * C + k], vy = st.A1l[Lp][j * 3 * C + C + k],
                    vz = st.A1l[Lp][j * 3 * C + 2 * C + k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float db0 = m.s[g][k];
        const float bx = m.v[g * 3][k], by = m.v[g * 3 + 1][k], bz = m.v[g * 3 + 2][k];
        float ga = db0 * (((p0[0] + 2.f * p0[C] * aa) + 3.f * p0[3 * C] * aa * aa) + p0[4 * C] * q);
        float gq = db0 * (p0[2 * C] + p0[4 * C] * aa);
        const float cc = ((p1[0] + p1[C] * aa) + p1[2 * C] * aa * aa) + p1[3 * C] * q;
        const float bv = (bx * vx + by * vy) + bz * vz;
        ga += bv * (p1[C] + 2.f * p1[2 * C] * aa);
        gq += bv * p1[3 * C];
        __syncthreads();
        m.s[g][k] = ga;
        m.v[g * 3][k] = cc * bx + 2.f * gq * vx;
        m.v[g * 3 + 1][k] = cc * by + 2.f * gq * vy;
        m.v[g * 3 + 2][k] = cc * bz + 2.f * gq * vz;
        __syncthreads();
        mix_rows<C, G, 3 * G>(m.s, w.lin0[Lp], m.v, w.lin1[Lp], m.s, m.v, m.red);
        if (my >= 0) {
            st.dA0[Lp][my * int64_t(C) + k] = m.s[g][k];
#pragma unroll
            for (int c = 0; c < 3; ++c) st.dA1[Lp][my * int64_t(3 * C) + c * C + k] = m.v[g * 3 + c][k];
        }
    }
}

// ------------------------------------------------- node path on the tensor cores
//
// For the large replica unions (the tensor-core radial path) of a 2-layer model, every
// element-independent channel mixing of the node kernels (lin, out and up, forward and backward: a
// [rows x C] x [C x C] product over all atoms, the scalar rows and the 3 vector rows of each atom as the
// two problems of one fmd_gemm_tf32x3_grouped launch) runs on the tensor cores; the per-element work
// stays on the CUDA cores in these kernels: the symmetric contraction and its backward (thread per atom
// and channel), and, per group of same-element atoms, the skip mixings, the readout and the sender
// gather. Each kernel's arithmetic is its node kernel's.

// b[i][k] (and bv[i][c][k] = cc v[i][c][k] when bv is given) of the symmetric contraction of layer L
template <int C>
__global__ void __launch_bounds__(256) tcn_contract_kernel(FusedWeights w, FusedState st, int L,
                                                           const float* __restrict__ a0l,
                                                           const float* __restrict__ a1l, float* __restrict__ b,
                                                           float* __restrict__ bv, int64_t n) {
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n * C;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = idx / C;
        const int k = int(idx % C);
        const int64_t z = st.elem[i];
        const float aa = a0l[i * C + k];
        const float vx = a1l[i * 3 * C + k], vy = a1l[i * 3 * C + C + k], vz = a1l[i * 3 * C + 2 * C + k];
        const float* p0 = w.prod0[L] + z * 5 * C + k;
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float b0 = (((p0[0] * aa + p0[C] * aa * aa) + p0[2 * C] * q) + p0[3 * C] * aa * aa * aa) + p0[4 * C] * aa * q;
        b[i * C + k] = b0;
        if (bv != nullptr) {
            const float* p1 = w.prod1[L] + z * 4 * C + k;
            const float cc = ((p1[0] + p1[C] * aa) + p1[2 * C] * aa * aa) + p1[3 * C] * q;
            bv[i * 3 * C + k] = cc * vx;
            bv[i * 3 * C + C + k] = cc * vy;
            bv[i * 3 * C + 2 * C + k] = cc * vz;
        }
    }
}

// dst[r] = src[order[r]] (rows of C floats): the rows in element order for the per-element GEMMs
template <int C>
__global__ void __launch_bounds__(256) tcn_gather_rows_kernel(const float* __restrict__ src,
                                                              const int32_t* __restrict__ order, int64_t n,
                                                              float* __restrict__ dst) {
    constexpr int V = C / 4;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n * V;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = idx / V;
        const int q = int(idx % V);
        reinterpret_cast<float4*>(dst + r * C)[q] = reinterpret_cast<const float4*>(src + int64_t(order[r]) * C)[q];
    }
}

// last layer, before its output mixing: t = the skip mixing of s_out[L - 1] (per element) into t_out, the
// layer-0 readout term e_term0 = s_out[0] . r0 (L = 1), and the scalar contraction b0 into b; with tp, the
// skip mixing was done by the per-element GEMMs in element order (row elem_rank[i] of tp) and is copied
template <int C, int G>
__global__ void __launch_bounds__(kQ * C, 2) tcn_last_pre_kernel(FusedWeights w, FusedState st, int L,
                                                                 float* __restrict__ t_out, float* __restrict__ b,
                                                                 const float* __restrict__ tp) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    NodeSmem<C>& m = *reinterpret_cast<NodeSmem<C>*>(smem_raw);
    const int k = threadIdx.x % C, g = threadIdx.x / C;
    for (int64_t grp = blockIdx.x; grp < node_units<G>(st); grp += gridDim.x) {
        int atoms[kG];
        group_atoms<G>(st, grp, atoms);
        if (atoms[0] < 0) continue;
        const int64_t z = st.elem[atoms[0]];
        const int my = atoms[g];
        const int64_t i = my < 0 ? atoms[0] : my;
        __syncthreads();
        m.t[g][k] = st.s_out[L - 1][i * C + k];
        __syncthreads();
        if (L - 1 == 0) {  // layer 0's readout, from its output (node_fwd's atom_sum)
            const float e = atom_sum<C>(m.t[g][k] * w.r0[k], m.sc);
            if (k == 0 && my >= 0) st.e_term0[my] = e;
        }
        if (tp == nullptr) mix_rows<C, G, 0>(m.t, w.skip0[L] + z * C * C, nullptr, nullptr, m.t, nullptr, m.red);
        const float aa = st.A0l[L][i * C + k];
        const float vx = st.A1l[L][i * 3 * C + k], vy = st.A1l[L][i * 3 * C + C + k],
                    vz = st.A1l[L][i * 3 * C + 2 * C + k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float* p0 = w.prod0[L] + z * 5 * C + k;
        const float b0 = (((p0[0] * aa + p0[C] * aa * aa) + p0[2 * C] * q) + p0[3 * C] * aa * aa * aa) + p0[4 * C] * aa * q;
        if (my >= 0) {
            t_out[my * int64_t(C) + k] = tp != nullptr ? tp[int64_t(st.elem_rank[my]) * C + k] : m.t[g][k];
            b[my * int64_t(C) + k] = b0;
        }
    }
}

// last layer, after its output mixing (so = s_out[L], the skip added by the GEMM): the readout MLP, the
// node energies, ds = dE/d so into ds_out and the skip backward into ds_skip[L]; with dsp, ds also into
// row elem_rank[i] of dsp for the per-element GEMMs, which do the skip backward instead
template <int C, int G>
__global__ void __launch_bounds__(kQ * C, 2) tcn_last_post_kernel(FusedWeights w, FusedState st, int L,
                                                                  float* __restrict__ ds_out,
                                                                  float* __restrict__ dsp) {
    static_assert((C & (C - 1)) == 0 && C >= 32, "the readout's channel rotation wraps with a mask");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    NodeSmem<C>& m = *reinterpret_cast<NodeSmem<C>*>(smem_raw);
    const int k = threadIdx.x % C, g = threadIdx.x / C;
    const int RH = w.readout_hidden;
    for (int idx = threadIdx.x; idx < RH * C; idx += kQ * C) m.ra[idx / C][idx % C] = w.ra[idx];
    for (int64_t grp = blockIdx.x; grp < node_units<G>(st); grp += gridDim.x) {
        int atoms[kG];
        group_atoms<G>(st, grp, atoms);
        if (atoms[0] < 0) continue;
        const int64_t z = st.elem[atoms[0]];
        const int my = atoms[g];
        const int64_t i = my < 0 ? atoms[0] : my;
        __syncthreads();
        m.s[g][k] = st.s_out[L][i * C + k];
        __syncthreads();
        // pre_j = s . ra_j: with RH = 16, thread (atom, j, eighth of the channels) sums C / 8 channels (walked
        // from a start that keeps a warp's reads on distinct banks), then a 3-step shuffle over the eighths;
        // otherwise thread (atom, j) walks all channels from c = j on
        if (RH == 16 && kQ * C >= kG * 16 * 8) {
            constexpr int CE = C / 8;
            const int gg = threadIdx.x / 128, j = (threadIdx.x >> 3) & 15, part = threadIdx.x & 7;
            float acc = 0.f;
            if (gg < G) {
                for (int cc = 0; cc < CE; ++cc) {
                    const int c = part * CE + ((cc + j + 4 * (part >> 1)) & (CE - 1));
                    acc = fmaf(m.s[gg][c], m.ra[j][c], acc);
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 4);
            if (part == 0 && gg < G) m.pre[gg][j] = acc;
        } else {
            for (int idx = threadIdx.x; idx < G * RH; idx += kQ * C) {
                const int gg = idx / RH, j = idx % RH;
                float acc = 0.f;
                for (int cc = 0; cc < C; ++cc) {
                    const int c = (cc + j) & (C - 1);
                    acc = fmaf(m.s[gg][c], m.ra[j][c], acc);
                }
                m.pre[gg][j] = acc;
            }
        }
        __syncthreads();
        // the energy (thread (atom, 0)) and the readout backward's coefficients rb_j silu'(pre_j), once per
        // (atom, j)
        if (k == 0 && my >= 0) {
            float e1 = 0.f;
            for (int j = 0; j < RH; ++j) e1 = fmaf(w.rb[j], silu_f(m.pre[g][j]), e1);
            st.node_energy[my] = w.e0[z] + w.scale * (double(st.e_term0[my]) + double(e1)) + w.shift;
        }
        if (k < RH) m.sc[g][k] = w.rb[k] * silu_g(m.pre[g][k]);
        __syncthreads();
        const float sc = float(w.scale);
        float acc = 0.f;
        for (int j = 0; j < RH; ++j) acc = fmaf(m.sc[g][j], m.ra[j][k], acc);
        const float ds = sc * acc;
        __syncthreads();
        if (dsp != nullptr) {
            if (my >= 0) {
                dsp[int64_t(st.elem_rank[my]) * C + k] = ds;
                ds_out[my * int64_t(C) + k] = ds;
            }
            continue;
        }
        m.t[g][k] = ds;
        __syncthreads();
        mix_rows<C, G, 0>(m.t, w.skip0t[L] + z * C * C, nullptr, nullptr, m.v, nullptr, m.red);
        if (my >= 0) {
            st.ds_skip[L][my * int64_t(C) + k] = m.v[g][k];
            ds_out[my * int64_t(C) + k] = ds;
        }
    }
}

// last layer, the contraction backward: from db0 (the output mixing's backward) to the lin mixing's
// input gradients (s: da, v: 2 gq v), in place over db0 / into gv
template <int C>
__global__ void __launch_bounds__(256) tcn_last_bwd_kernel(FusedWeights w, FusedState st, int L,
                                                           float* __restrict__ db, float* __restrict__ gv,
                                                           const float* __restrict__ dskp, int64_t n) {
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n * C;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = idx / C;
        const int k = int(idx % C);
        const int64_t z = st.elem[i];
        const float aa = st.A0l[L][i * C + k];
        const float vx = st.A1l[L][i * 3 * C + k], vy = st.A1l[L][i * 3 * C + C + k],
                    vz = st.A1l[L][i * 3 * C + 2 * C + k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float* p0 = w.prod0[L] + z * 5 * C + k;
        const float db0 = db[i * C + k];
        const float gq = db0 * (p0[2 * C] + p0[4 * C] * aa);
        const float da = db0 * (((p0[0] + 2.f * p0[C] * aa) + 3.f * p0[3 * C] * aa * aa) + p0[4 * C] * q);
        db[i * C + k] = da;
        if (dskp != nullptr) st.ds_skip[L][i * C + k] = dskp[int64_t(st.elem_rank[i]) * C + k];
        gv[i * 3 * C + k] = 2.f * gq * vx;
        gv[i * 3 * C + C + k] = 2.f * gq * vy;
        gv[i * 3 * C + 2 * C + k] = 2.f * gq * vz;
    }
}

// the sender side of layer L: each atom's gathered edge gradient (the first phase of sender_node) into
// gs [N][C] and gv [N][3][C]
template <int C, int G>
__global__ void __launch_bounds__(kQ * C, 2) tcn_sender_gather_kernel(GraphArgs gr, FusedWeights w, FusedState st,
                                                                      int L, float* __restrict__ gs,
                                                                      float* __restrict__ gv) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    NodeSmem<C>& m = *reinterpret_cast<NodeSmem<C>*>(smem_raw);
    constexpr int CPL = C / 32, NW = C / 32;
    const int k = threadIdx.x % C, g = threadIdx.x / C;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ga = warp / NW, wa = warp % NW;
    float (*redf)[C] = reinterpret_cast<float (*)[C]>(&m.red[0][0][0]);
    const int P = 4;
    const float* R = st.R[L];
    for (int64_t grp = blockIdx.x; grp < node_units<G>(st); grp += gridDim.x) {
        int atoms[kG];
        group_atoms<G>(st, grp, atoms);
        if (atoms[0] < 0) continue;
        const int my = atoms[g];
        const int mw = atoms[ga];
        const int64_t jw = mw < 0 ? atoms[0] : mw;
        float ds[CPL], dx[CPL], dy[CPL], dz[CPL];
#pragma unroll
        for (int qq = 0; qq < CPL; ++qq) ds[qq] = dx[qq] = dy[qq] = dz[qq] = 0.f;
        for (int64_t t = gr.send_off[jw] + wa; ga < G && t < gr.send_off[jw + 1]; t += NW) {
            const int64_t e = gr.send_perm[t];
            const int64_t i = gr.edge_index[2 * e];
            const float4 y = st.ysh[e];
            const float* Re = R + e * (P * C) + lane * CPL;
            const float* a0 = st.dA0[L] + i * C + lane * CPL;
            const float* a1 = st.dA1[L] + i * 3 * C + lane * CPL;
            float r0[CPL], r1[CPL], r2v[CPL], r3v[CPL], d0[CPL], dxv[CPL], dyv[CPL], dzv[CPL];
            ldv<CPL>(Re, r0);
            ldv<CPL>(Re + C, r1);
            ldv<CPL>(Re + 2 * C, r2v);
            ldv<CPL>(Re + 3 * C, r3v);
            ldv<CPL>(a0, d0);
            ldv<CPL>(a1, dxv);
            ldv<CPL>(a1 + C, dyv);
            ldv<CPL>(a1 + 2 * C, dzv);
#pragma unroll
            for (int qq = 0; qq < CPL; ++qq) {
                const float g0 = d0[qq] * w.inv_avg;
                const float gx = dxv[qq] * w.inv_avg;
                const float gy = dyv[qq] * w.inv_avg;
                const float gz = dzv[qq] * w.inv_avg;
                ds[qq] = fmaf(r0[qq], g0, ds[qq]);
                ds[qq] = fmaf(r1[qq], (gx * y.x + gy * y.y) + gz * y.z, ds[qq]);
                const float r2 = r2v[qq], r3 = r3v[qq] * g0 * kIS3;
                dx[qq] = fmaf(r2, gx, fmaf(r3, y.x, dx[qq]));
                dy[qq] = fmaf(r2, gy, fmaf(r3, y.y, dy[qq]));
                dz[qq] = fmaf(r2, gz, fmaf(r3, y.z, dz[qq]));
            }
        }
        __syncthreads();
#pragma unroll
        for (int qq = 0; qq < CPL; ++qq) {
            const int kk = lane * CPL + qq;
            redf[(ga * NW + wa) * 4 + 0][kk] = ds[qq];
            redf[(ga * NW + wa) * 4 + 1][kk] = dx[qq];
            redf[(ga * NW + wa) * 4 + 2][kk] = dy[qq];
            redf[(ga * NW + wa) * 4 + 3][kk] = dz[qq];
        }
        __syncthreads();
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
        if (g < G)
            for (int wv = 0; wv < NW; ++wv)
#pragma unroll
                for (int c = 0; c < 4; ++c) sum[c] += redf[(g * NW + wv) * 4 + c][k];
        if (my >= 0) {
            gs[my * int64_t(C) + k] = sum[0];
#pragma unroll
            for (int c = 0; c < 3; ++c) gv[my * int64_t(3 * C) + c * C + k] = sum[1 + c];
        }
    }
}

// between the up-mixing backward and the output mixing backward of layer Lp = L - 1 (in place): the skip
// connection's gradient and the layer-0 readout
template <int C>
__global__ void __launch_bounds__(256) tcn_sender_mid_kernel(FusedWeights w, FusedState st, int L,
                                                             float* __restrict__ s, float* __restrict__ v, int64_t n) {
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n * C;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = idx / C;
        const int k = int(idx % C);
        float dsi = s[i * C + k];
        if (st.ds_skip[L]) dsi += st.ds_skip[L][i * C + k];
        if (L - 1 == 0) dsi = fmaf(float(w.scale), w.r0[k], dsi);
        s[i * C + k] = dsi;
        if (st.dv_skip[L])
#pragma unroll
            for (int c = 0; c < 3; ++c) v[i * 3 * C + c * C + k] += st.dv_skip[L][i * 3 * C + c * C + k];
    }
}

// the product backward of layer Lp (in place): from (db0, b) to (ga, cc b + 2 gq v)
template <int C>
__global__ void __launch_bounds__(256) tcn_sender_prod_kernel(FusedWeights w, FusedState st, int Lp,
                                                              float* __restrict__ s, float* __restrict__ v,
                                                              int64_t n) {
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < n * C;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = idx / C;
        const int k = int(idx % C);
        const int64_t z = st.elem[i];
        const float* p0 = w.prod0[Lp] + z * 5 * C + k;
        const float* p1 = w.prod1[Lp] + z * 4 * C + k;
        const float aa = st.A0l[Lp][i * C + k];
        const float vx = st.A1l[Lp][i * 3 * C + k], vy = st.A1l[Lp][i * 3 * C + C + k],
                    vz = st.A1l[Lp][i * 3 * C + 2 * C + k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float db0 = s[i * C + k];
        const float bx = v[i * 3 * C + k], by = v[i * 3 * C + C + k], bz = v[i * 3 * C + 2 * C + k];
        float ga = db0 * (((p0[0] + 2.f * p0[C] * aa) + 3.f * p0[3 * C] * aa * aa) + p0[4 * C] * q);
        float gq = db0 * (p0[2 * C] + p0[4 * C] * aa);
        const float cc = ((p1[0] + p1[C] * aa) + p1[2 * C] * aa * aa) + p1[3 * C] * q;
        const float bv = (bx * vx + by * vy) + bz * vz;
        ga += bv * (p1[C] + 2.f * p1[2 * C] * aa);
        gq += bv * p1[3 * C];
        s[i * C + k] = ga;
        v[i * 3 * C + k] = cc * bx + 2.f * gq * vx;
        v[i * 3 * C + C + k] = cc * by + 2.f * gq * vy;
        v[i * 3 * C + 2 * C + k] = cc * bz + 2.f * gq * vz;
    }
}

// ---------------------------------------------------------------- edge backward

constexpr int kBT = 512;        // threads of the backward edge kernel
constexpr int kBQ = kBT / kH;   // column blocks of dR . W4 (thread (k, block))

struct EdgeBwdSmem {
    float phi[kTB][16];
    float dphi[kTB][16];
    float h[2][kTB][kHS];       // h1, h2 (post-activation)
    float p[3][kTB][kHS];       // pre-activations
    float g[2][kTB][kHS];       // gradient ping-pong
    float w1[16][kH];
    float w2[kH][kWS];
    float w3[kH][kWS];
    float dR[kTB][kMaxPC];      // the tile's dR rows
    float red[kBQ][kTB][kH];    // partials of dR . W4 over kBQ column blocks
};

// dh3[e][k] = sum_n dR[e][n] W4[n][k]: thread (k, block of n), float4 broadcast reads of dR
template <int PC>
__device__ __forceinline__ void radial_out_bwd(const float (*dR)[kMaxPC], const float* __restrict__ W4,
                                               float (*red)[kTB][kH]) {
    constexpr int NQ = PC / kBQ;
    const int k = threadIdx.x % kH, qt = threadIdx.x / kH;
    float acc[kTB];
#pragma unroll
    for (int e = 0; e < kTB; ++e) acc[e] = 0.f;
#pragma unroll 4
    for (int nn = 0; nn < NQ; nn += 4) {
        const int n = qt * NQ + nn;
        const float w0 = W4[(n + 0) * kH + k], w1 = W4[(n + 1) * kH + k];
        const float w2 = W4[(n + 2) * kH + k], w3 = W4[(n + 3) * kH + k];
#pragma unroll
        for (int e = 0; e < kTB; ++e) {
            const float4 x = *reinterpret_cast<const float4*>(&dR[e][n]);
            acc[e] = fmaf(x.x, w0, fmaf(x.y, w1, fmaf(x.z, w2, fmaf(x.w, w3, acc[e]))));
        }
    }
#pragma unroll
    for (int e = 0; e < kTB; ++e) red[qt][e][k] = acc[e];
}

// stage the tile's dR rows (float4, unrolled)
template <int PC>
__device__ __forceinline__ void stage_dr(float (*dst)[kMaxPC], const float* __restrict__ dR, int64_t e0, int ne) {
    constexpr int V = (kTB * PC / 4 + kBT - 1) / kBT;  // float4 per thread (the last round partial)
#pragma unroll
    for (int r = 0; r < V; ++r) {
        const int idx = threadIdx.x + kBT * r;
        if (idx >= kTB * PC / 4) break;
        const int e = (idx * 4) / PC, n = (idx * 4) % PC;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < ne) v = reinterpret_cast<const float4*>(dR + (e0 + e) * PC)[n / 4];
        *reinterpret_cast<float4*>(&dst[e][n]) = v;
    }
}

// out[e][k] = (sum_c g[e][c] W[k][c]) * silu'(pre[e][k]) (the transpose walk of a staged W^T)
__device__ __forceinline__ void hidden_bwd(const float (*g)[kHS], const float (*W)[kWS], const float (*pre)[kHS],
                                           float (*out)[kHS]) {
    constexpr int EPG = kTB / kBQ;
    const int k = threadIdx.x % kH, eg = threadIdx.x / kH;
    float acc[EPG];
#pragma unroll
    for (int m = 0; m < EPG; ++m) acc[m] = 0.f;
#pragma unroll 4
    for (int c = 0; c < kH; c += 4) {
        const float w0 = W[k][c], w1 = W[k][c + 1], w2 = W[k][c + 2], w3 = W[k][c + 3];
#pragma unroll
        for (int m = 0; m < EPG; ++m) {
            const float4 x = *reinterpret_cast<const float4*>(&g[eg * EPG + m][c]);
            acc[m] = fmaf(x.x, w0, fmaf(x.y, w1, fmaf(x.z, w2, fmaf(x.w, w3, acc[m]))));
        }
    }
#pragma unroll
    for (int m = 0; m < EPG; ++m) out[eg * EPG + m][k] = acc[m] * silu_g(pre[eg * EPG + m][k]);
}

// g_r[e] = dE/dr_e from the spherical-harmonic gradient dY[e] and the radial-feature gradient dphi
// (the geometry backward of one edge)
__device__ __forceinline__ void geometry_grad(const FusedWeights& w, const FusedState& st, int64_t e,
                                              const float* dphi) {
    const float pref = sqrtf(2.0f / w.r_max);
    const float4 y = st.ysh[e];
    const float d = y.w;
    float gx = 0.f, gy = 0.f, gz = 0.f;
    if (d > 0.f) {
        const float inv = 1.0f / d;
        const float ux = y.x * kIS3, uy = y.y * kIS3, uz = y.z * kIS3;
        const float* gyv = st.dY + 3 * e;
        const float gu = (gyv[0] * ux + gyv[1] * uy) + gyv[2] * uz;
        gx = kS3 * (gyv[0] - gu * ux) * inv;
        gy = kS3 * (gyv[1] - gu * uy) * inv;
        gz = kS3 * (gyv[2] - gu * uz) * inv;
        float f, df;
        cutoff_poly(d, w.r_max, w.poly_p, f, df);
        float gd = 0.f;
        for (int n = 0; n < w.n_basis; ++n) {
            const float k = float(n + 1) * 3.14159265358979323846f / w.r_max;
            float sn, cs;
            sincosf(k * d, &sn, &cs);
            const float b = pref * sn * inv;
            const float db = pref * (k * cs * d - sn) * inv * inv;
            gd += dphi[n] * (db * f + b * df);
        }
        gx += gd * ux;
        gy += gd * uy;
        gz += gd * uz;
    }
    st.g_r[3 * e] = gx;
    st.g_r[3 * e + 1] = gy;
    st.g_r[3 * e + 2] = gz;
}

// the radial MLP backward of every layer (the forward recomputed from the distances) and the
// geometry backward: g_r [E][3] = dE/dr_e
template <int C>
__global__ void __launch_bounds__(kBT) edge_bwd_kernel(EdgeArgs a, FusedWeights w, FusedState st) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    EdgeBwdSmem& m = *reinterpret_cast<EdgeBwdSmem*>(smem_raw);
    const int t = threadIdx.x;
    const float pref = sqrtf(2.0f / w.r_max);
    const int64_t n_edges = real_edges(a);
    const int64_t n_tiles = (n_edges + kTB - 1) / kTB;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t e0 = tile * kTB;
        const int ne = int(n_edges - e0 < kTB ? n_edges - e0 : kTB);
        __syncthreads();
        if (t < kTB) {
            const float d = t < ne ? st.ysh[e0 + t].w : 0.f;
            float f, df;
            cutoff_poly(d, w.r_max, w.poly_p, f, df);
            const float inv = d > 0.f ? 1.0f / d : 0.f;
            for (int n = 0; n < w.n_basis; ++n) {
                const float k = float(n + 1) * 3.14159265358979323846f / w.r_max;
                m.phi[t][n] = d > 0.f ? pref * sinf(k * d) * inv * f : 0.f;
                m.dphi[t][n] = 0.f;
            }
        }
        for (int L = 0; L < w.n_layers; ++L) {
            __syncthreads();
            stage_radial<kBT>(m.w1, m.w2, m.w3, w, L);
            if (L == 0) stage_dr<2 * C>(m.dR, st.dR[L], e0, ne);
            else stage_dr<4 * C>(m.dR, st.dR[L], e0, ne);
            __syncthreads();
            // forward recompute
            for (int idx = t; idx < kTB * kH; idx += kBT) {
                const int e = idx / kH, k = idx % kH;
                float acc = 0.f;
                for (int n = 0; n < w.n_basis; ++n) acc = fmaf(m.phi[e][n], m.w1[n][k], acc);
                m.p[0][e][k] = acc;
                m.h[0][e][k] = silu_f(acc);
            }
            __syncthreads();
            hidden_layer<kTB, true, kBT>(m.h[0], m.w2, m.h[1], m.p[1]);
            __syncthreads();
            hidden_layer<kTB, false, kBT>(m.h[1], m.w3, m.g[1], m.p[2]);  // only the pre-activation is kept
            if (L == 0) radial_out_bwd<2 * C>(m.dR, w.w4[L], m.red);
            else radial_out_bwd<4 * C>(m.dR, w.w4[L], m.red);
            __syncthreads();
            for (int idx = t; idx < kTB * kH; idx += kBT) {
                const int e = idx / kH, k = idx % kH;
                float part[kBQ];
#pragma unroll
                for (int b = 0; b < kBQ; ++b) part[b] = m.red[b][e][k];
#pragma unroll
                for (int width = kBQ / 2; width > 0; width /= 2)
#pragma unroll
                    for (int b = 0; b < width; ++b) part[b] = part[b] + part[b + width];
                m.g[0][e][k] = part[0] * silu_g(m.p[2][e][k]);
            }
            __syncthreads();
            hidden_bwd(m.g[0], m.w3, m.p[1], m.g[1]);
            __syncthreads();
            hidden_bwd(m.g[1], m.w2, m.p[0], m.g[0]);
            __syncthreads();
            // dphi += g1 . W1 (W1[c][n] = W1^T[n][c])
            for (int idx = t; idx < kTB * w.n_basis; idx += kBT) {
                const int e = idx / w.n_basis, n = idx % w.n_basis;
                float acc = 0.f;
#pragma unroll 16
                for (int c = 0; c < kH; ++c) acc = fmaf(m.g[0][e][c], m.w1[n][c], acc);
                m.dphi[e][n] += acc;
            }
        }
        __syncthreads();
        if (t < ne) geometry_grad(w, st, e0 + t, m.dphi[t]);
    }
}

// ------------------------------------------------ tensor-core radial MLP path

constexpr int kTG = 64;  // edges per tile of the geometry kernels (256 threads: geometry per edge, basis
                         // functions and the first-layer products spread over the CTA)

// geometry, radial features and the first radial layer's pre-activation p1 = phi W1^T of every layer
// for every edge row (padding rows after the real count: p1 = 0, so the GEMM chain yields R = 0 there)
__global__ void __launch_bounds__(256) edge_geom_tc_kernel(EdgeArgs a, FusedWeights w, FusedState st) {
    __shared__ float phi[kTG][17];
    __shared__ float geo[kTG][3];  // d, 1 / d, cutoff envelope f
    __shared__ __align__(16) float w1t[kMaxLayers][16][kH];
    const int t = threadIdx.x;
    const float pref = sqrtf(2.0f / w.r_max);
    const int64_t n_real = real_edges(a);
    for (int L = 0; L < w.n_layers; ++L)
        for (int idx = t; idx < w.n_basis * kH; idx += 256) w1t[L][idx / kH][idx % kH] = w.w1t[L][idx];
    const int64_t n_tiles = (a.n_edges + kTG - 1) / kTG;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t e0 = tile * kTG;
        const int ne = int(a.n_edges - e0 < kTG ? a.n_edges - e0 : kTG);
        __syncthreads();
        if (t < kTG) {
            const int64_t e = e0 + t;
            float d = 0.f;
            if (e < n_real) {
                const int64_t i = a.edge_index[2 * e], j = a.edge_index[2 * e + 1];
                const float ix = a.edge_image[3 * e], iy = a.edge_image[3 * e + 1], iz = a.edge_image[3 * e + 2];
                const float* c = a.cell;
                const float rx = (a.pos[3 * j] - a.pos[3 * i]) + ((ix * c[0] + iy * c[3]) + iz * c[6]);
                const float ry = (a.pos[3 * j + 1] - a.pos[3 * i + 1]) + ((ix * c[1] + iy * c[4]) + iz * c[7]);
                const float rz = (a.pos[3 * j + 2] - a.pos[3 * i + 2]) + ((ix * c[2] + iy * c[5]) + iz * c[8]);
                d = sqrtf((rx * rx + ry * ry) + rz * rz);
                const float inv = d > 0.f ? 1.0f / d : 0.f;
                st.ysh[e] = make_float4(kS3 * rx * inv, kS3 * ry * inv, kS3 * rz * inv, d);
            }
            float f, df;
            cutoff_poly(d, w.r_max, w.poly_p, f, df);
            geo[t][0] = d;
            geo[t][1] = d > 0.f ? 1.0f / d : 0.f;
            geo[t][2] = f;
        }
        __syncthreads();
        for (int idx = t; idx < kTG * w.n_basis; idx += 256) {
            const int e = idx / w.n_basis, n = idx % w.n_basis;
            const float d = geo[e][0];
            const float k = float(n + 1) * 3.14159265358979323846f / w.r_max;
            phi[e][n] = d > 0.f ? pref * sinf(k * d) * geo[e][1] * geo[e][2] : 0.f;
        }
        __syncthreads();
        // p1[e][k] = sum_n phi[e][n] W1^T[n][k] in n order: thread (edge, 4 channels) holds the edge's basis in
        // registers and reads W1^T four channels per 16-byte broadcast, stores four channels per float4
        for (int L = 0; L < w.n_layers; ++L) {
            float* p1 = st.pre[0][L];
            for (int idx = t; idx < ne * (kH / 4); idx += 256) {
                const int e = idx / (kH / 4), k = (idx % (kH / 4)) * 4;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int n = 0; n < w.n_basis; ++n) {
                    const float ph = phi[e][n];
                    const float4 wv = *reinterpret_cast<const float4*>(&w1t[L][n][k]);
                    acc.x = fmaf(ph, wv.x, acc.x);
                    acc.y = fmaf(ph, wv.y, acc.y);
                    acc.z = fmaf(ph, wv.z, acc.z);
                    acc.w = fmaf(ph, wv.w, acc.w);
                }
                *reinterpret_cast<float4*>(p1 + (e0 + e) * kH + k) = acc;
            }
        }
    }
}

// dphi = sum over layers of g1 W1 (g1 = dE/dp1, left in the p1 buffer by the GEMM chain), then the
// geometry backward of every real edge
__global__ void __launch_bounds__(256) edge_geom_bwd_tc_kernel(EdgeArgs a, FusedWeights w, FusedState st) {
    __shared__ __align__(16) float w1[kMaxLayers][kH][16];  // W1 [hidden][basis]
    __shared__ float g[kTG][kH + 1];
    __shared__ float dphi[kTG][16];
    const int t = threadIdx.x;
    const int nb = w.n_basis;
    for (int L = 0; L < w.n_layers; ++L)
        for (int idx = t; idx < kH * 16; idx += 256) {
            const int c = idx / 16, n = idx % 16;
            w1[L][c][n] = n < nb ? w.w1[L][c * nb + n] : 0.f;
        }
    const int64_t n_edges = real_edges(a);
    const int64_t n_tiles = (n_edges + kTG - 1) / kTG;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t e0 = tile * kTG;
        const int ne = int(n_edges - e0 < kTG ? n_edges - e0 : kTG);
        __syncthreads();
        for (int idx = t; idx < kTG * 16; idx += 256) dphi[idx / 16][idx % 16] = 0.f;
        for (int L = 0; L < w.n_layers; ++L) {
            const float* g1 = st.pre[0][L];
            __syncthreads();
            for (int idx = t; idx < ne * kH; idx += 256) g[idx / kH][idx % kH] = g1[(e0 + idx / kH) * kH + idx % kH];
            __syncthreads();
            // dphi[e][n] += sum_c g[e][c] W1[c][n] in c order: thread (edge, 4 basis functions), the W1 row read
            // four basis functions per 16-byte broadcast
            for (int idx = t; idx < ne * 4; idx += 256) {
                const int e = idx >> 2, n0 = (idx & 3) * 4;
                if (n0 >= nb) continue;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
                for (int c = 0; c < kH; ++c) {
                    const float gv = g[e][c];
                    const float4 wv = *reinterpret_cast<const float4*>(&w1[L][c][n0]);
                    acc.x = fmaf(gv, wv.x, acc.x);
                    acc.y = fmaf(gv, wv.y, acc.y);
                    acc.z = fmaf(gv, wv.z, acc.z);
                    acc.w = fmaf(gv, wv.w, acc.w);
                }
                dphi[e][n0] += acc.x;
                if (n0 + 1 < nb) dphi[e][n0 + 1] += acc.y;
                if (n0 + 2 < nb) dphi[e][n0 + 2] += acc.z;
                if (n0 + 3 < nb) dphi[e][n0 + 3] += acc.w;
            }
        }
        __syncthreads();
        if (t < ne) geometry_grad(w, st, e0 + t, dphi[t]);
    }
}

// the radial MLPs of every layer as GEMMs on the tensor cores:
//   p2 = silu(p1) W2^T, p3 = silu(p2) W3^T, R = silu(p3) W4^T
fmd_status radial_tc_forward(const FusedWeights& w, const FusedState& st, int64_t E, int C, cudaStream_t s) {
    // the layers' chains are independent: GEMM k of every layer in one grouped launch (bitwise the
    // single calls), 3 launches instead of 3 per layer
    for (int k = 0; k < 3; ++k) {
        fmd_gemm_problem pr[kMaxLayers];
        for (int L = 0; L < w.n_layers; ++L) {
            const int PC = (L == 0 ? 2 : 4) * C;
            const int n = k < 2 ? kH : PC;
            pr[L] = fmd_gemm_problem{st.pre[k][L], kH, w.tc_hi[k][L], w.tc_lo[k][L], kH, nullptr, nullptr, 0,
                                     k < 2 ? st.pre[k + 1][L] : st.R[L], n, E, n, kH,
                                     FMD_ACT_NONE | FMD_ACT_INPUT_SILU, 0};
        }
        const fmd_status r = fmd_gemm_tf32x3_grouped(pr, w.n_layers, st.flags, s);
        if (r != FMD_OK) return r;
    }
    return FMD_OK;
}

// their backward, each gradient written over its pre-activation:
//   g3 = (dR W4) silu'(p3), g2 = (g3 W3) silu'(p2), g1 = (g2 W2) silu'(p1)
// (GEMM k of every layer in one grouped launch, as the forward)
fmd_status radial_tc_backward(const FusedWeights& w, const FusedState& st, int64_t E, int C, cudaStream_t s) {
    for (int k = 2; k >= 0; --k) {
        fmd_gemm_problem pr[kMaxLayers];
        for (int L = 0; L < w.n_layers; ++L) {
            const int PC = (L == 0 ? 2 : 4) * C;
            const float* x = k == 2 ? st.dR[L] : st.pre[k + 1][L];
            const int K = k == 2 ? PC : kH;
            pr[L] = fmd_gemm_problem{x, K, w.tc_t_hi[k][L], w.tc_t_lo[k][L], K, nullptr, st.pre[k][L], kH,
                                     st.pre[k][L], kH, E, kH, K, FMD_ACT_SILU_GRAD, 0};
        }
        const fmd_status r = fmd_gemm_tf32x3_grouped(pr, w.n_layers, st.flags, s);
        if (r != FMD_OK) return r;
    }
    return FMD_OK;
}

// every pointer of the tensor-core path present, and the step large enough
bool use_radial_tc(const FusedWeights& w, const FusedState& st, int64_t n_edges) {
    if (w.tc_min_edges <= 0 || n_edges < w.tc_min_edges) return false;
    for (int L = 0; L < w.n_layers; ++L)
        for (int k = 0; k < 3; ++k)
            if (!w.tc_hi[k][L] || !w.tc_lo[k][L] || !w.tc_t_hi[k][L] || !w.tc_t_lo[k][L] || !st.pre[k][L])
                return false;
    return true;
}

// forces F_a = sum over received edges of g_r - sum over sent edges of g_r (a warp per atom: lanes over
// the atom's edges, a fixed xor tree over the lanes), and the per-system energy sums (the first CTA of
// each system, a fixed assignment of atoms to threads): grid (atom chunks, systems)
constexpr int kForceWarps = 8;
__global__ void __launch_bounds__(32 * kForceWarps) forces_kernel(GraphArgs g, const float* __restrict__ g_r,
                                                                  const double* __restrict__ node_energy,
                                                                  int64_t atoms_per_system, float* __restrict__ forces,
                                                                  double* __restrict__ total) {
    __shared__ double s_part[kForceWarps];
    const int64_t sys = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t la = int64_t(blockIdx.x) * kForceWarps + warp; la < atoms_per_system;
         la += int64_t(gridDim.x) * kForceWarps) {
        const int64_t a = sys * atoms_per_system + la;
        float fx = 0.f, fy = 0.f, fz = 0.f;
        for (int64_t e = g.recv_off[a] + lane; e < g.recv_off[a + 1]; e += 32) {
            fx += g_r[3 * e];
            fy += g_r[3 * e + 1];
            fz += g_r[3 * e + 2];
        }
        for (int64_t t = g.send_off[a] + lane; t < g.send_off[a + 1]; t += 32) {
            const int64_t e = g.send_perm[t];
            fx -= g_r[3 * e];
            fy -= g_r[3 * e + 1];
            fz -= g_r[3 * e + 2];
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            fx += __shfl_xor_sync(0xffffffffu, fx, d);
            fy += __shfl_xor_sync(0xffffffffu, fy, d);
            fz += __shfl_xor_sync(0xffffffffu, fz, d);
        }
        if (lane == 0) {
            forces[3 * a] = fx;
            forces[3 * a + 1] = fy;
            forces[3 * a + 2] = fz;
        }
    }
    if (blockIdx.x != 0) return;
    double acc_e = 0.0;
    for (int64_t la = threadIdx.x; la < atoms_per_system; la += blockDim.x)
        acc_e += node_energy[sys * atoms_per_system + la];
    for (int d = 16; d > 0; d >>= 1) acc_e += __shfl_xor_sync(0xffffffffu, acc_e, d);
    if (lane == 0) s_part[warp] = acc_e;
    __syncthreads();
    if (threadIdx.x == 0) {
        double sum = 0.0;
        for (int wv = 0; wv < kForceWarps; ++wv) sum += s_part[wv];
        total[sys] = sum;
    }
}

// the node path's channel mixings on the tensor cores: a 2-layer model with every split present
bool use_node_tc(const FusedWeights& w, bool radial_tc) {
    if (!radial_tc || w.n_layers != 2) return false;
    // layer 0: lin, out (both directions); layer 1 (the last): lin, out0, up (both directions)
    const int need0[8] = {0, 1, 2, 3, 6, 7, 8, 9};
    const int need1[10] = {0, 1, 2, 4, 5, 6, 7, 8, 10, 11};
    for (int m : need0)
        if (!w.ntc_hi[m][0] || !w.ntc_lo[m][0]) return false;
    for (int m : need1)
        if (!w.ntc_hi[m][1] || !w.ntc_lo[m][1]) return false;
    return true;
}

// ys = xs W_ms^T (+ cs) over the N scalar rows and yv = xv W_mv^T (+ cv) over the 3N vector rows of layer L's
// mixing m (one grouped launch; xv null: the scalar rows alone)
template <int C>
fmd_status node_mix(const FusedWeights& w, const FusedState& st, int64_t n, int L, int ms, int mv, const float* xs,
                    float* ys, const float* cs, const float* xv, float* yv, const float* cv, cudaStream_t s) {
    fmd_gemm_problem q[2] = {
        {xs, C, w.ntc_hi[ms][L], w.ntc_lo[ms][L], C, nullptr, cs, C, ys, C, n, C, C, 0, 0},
        {xv, C, w.ntc_hi[mv][L], w.ntc_lo[mv][L], C, nullptr, cv, C, yv, C, 3 * n, C, C, 0, 0}};
    return fmd_gemm_tf32x3_grouped(q, xv != nullptr ? 2 : 1, st.flags, s);
}

// y rows (element order) = the per-element skip mixing of x rows (element order) of layer L: direction d = 0
// the forward (skip0t), 1 the backward (skip0); one problem per element run, up to four per launch
template <int C>
fmd_status skip_mix(const FusedWeights& w, const FusedState& st, int L, int d, const float* x, float* y,
                    cudaStream_t s) {
    for (int64_t r0 = 0; r0 < st.n_runs; r0 += 4) {
        fmd_gemm_problem q[4];
        int np = 0;
        for (int64_t r = r0; r < st.n_runs && r < r0 + 4; ++r) {
            const int64_t z = st.runs_host[3 * r], first = st.runs_host[3 * r + 1], count = st.runs_host[3 * r + 2];
            q[np++] = {x + first * C, C, w.skip_hi[d][L] + z * C * C, w.skip_lo[d][L] + z * C * C, C, nullptr,
                       nullptr, 0, y + first * C, C, count, C, C, 0, 0};
        }
        const fmd_status r = fmd_gemm_tf32x3_grouped(q, np, st.flags, s);
        if (r != FMD_OK) return r;
    }
    return FMD_OK;
}

// node_fwd (L = 0), node_last (L = 1) and sender_node (L = 1) of a 2-layer model on the tensor-core path;
// the state buffers that are free at each point hold the intermediates
template <int C>
fmd_status node_tc_forward(const FusedWeights& w, const FusedState& st, int64_t n, int group_grid, bool single,
                           size_t node_smem, int L, cudaStream_t s) {
    const int eg = int((n * C + 255) / 256 < int64_t(kNumSMs) * 8 ? (n * C + 255) / 256 : int64_t(kNumSMs) * 8);
    fmd_status r = node_mix<C>(w, st, n, L, 0, 1, st.A0[L], st.A0l[L], nullptr, st.A1[L], st.A1l[L], nullptr, s);
    if (r != FMD_OK) return r;
    if (L == 0) {  // node_fwd: contraction, output mixing, the next layer's up-mixing
        tcn_contract_kernel<C><<<eg, 256, 0, s>>>(w, st, L, st.A0l[L], st.A1l[L], st.dA0[L], st.dA1[L], n);
        if ((r = check_launch()) != FMD_OK) return r;
        r = node_mix<C>(w, st, n, L, 2, 3, st.dA0[L], st.s_out[L], nullptr, st.dA1[L], st.v_out[L], nullptr, s);
        if (r != FMD_OK) return r;
        return node_mix<C>(w, st, n, L + 1, 4, 5, st.s_out[L], st.s_t[L + 1], nullptr, st.v_out[L], st.v_t[L + 1],
                           nullptr, s);
    }
    // node_last: skip and contraction (per element), output mixing + skip, readout and its backward, the
    // output mixing's backward, the contraction's backward, the lin mixing's backward
    float* t = st.A0[L];     // the skip term, then db0 and da
    float* b = st.dA0[L];    // b0
    float* dsb = st.v_out[L];  // ds (the first N C floats)
    // the skip mixings on the tensor cores when the atoms' element runs and the splits are given: rows in
    // element order in dA1[L] (free until the lin backward writes it), x / ds in its first N C floats, the
    // mixings' outputs in the next
    const bool tskip = w.skip_hi[0][L] && w.skip_lo[0][L] && w.skip_hi[1][L] && w.skip_lo[1][L] &&
                       st.elem_order && st.elem_rank && st.n_runs > 0 && st.runs_host;
    float* xp = st.dA1[L];
    float* yp = st.dA1[L] + n * C;
    if (tskip) {
        const int gg = int((n * C / 4 + 255) / 256 < int64_t(kNumSMs) * 8 ? (n * C / 4 + 255) / 256 : int64_t(kNumSMs) * 8);
        tcn_gather_rows_kernel<C><<<gg, 256, 0, s>>>(st.s_out[L - 1], st.elem_order, n, xp);
        if ((r = check_launch()) != FMD_OK) return r;
        if ((r = skip_mix<C>(w, st, L, 0, xp, yp, s)) != FMD_OK) return r;
    }
    if (single) tcn_last_pre_kernel<C, 1><<<group_grid, kQ * C, node_smem, s>>>(w, st, L, t, b, tskip ? yp : nullptr);
    else tcn_last_pre_kernel<C, kG><<<group_grid, kQ * C, node_smem, s>>>(w, st, L, t, b, tskip ? yp : nullptr);
    if ((r = check_launch()) != FMD_OK) return r;
    if ((r = node_mix<C>(w, st, n, L, 2, 3, b, st.s_out[L], t, nullptr, nullptr, nullptr, s)) != FMD_OK) return r;
    if (single) tcn_last_post_kernel<C, 1><<<group_grid, kQ * C, node_smem, s>>>(w, st, L, dsb, tskip ? xp : nullptr);
    else tcn_last_post_kernel<C, kG><<<group_grid, kQ * C, node_smem, s>>>(w, st, L, dsb, tskip ? xp : nullptr);
    if ((r = check_launch()) != FMD_OK) return r;
    if (tskip && (r = skip_mix<C>(w, st, L, 1, xp, yp, s)) != FMD_OK) return r;
    if ((r = node_mix<C>(w, st, n, L, 8, 9, dsb, t, nullptr, nullptr, nullptr, nullptr, s)) != FMD_OK) return r;
    tcn_last_bwd_kernel<C><<<eg, 256, 0, s>>>(w, st, L, t, st.A1[L], tskip ? yp : nullptr, n);
    if ((r = check_launch()) != FMD_OK) return r;
    return node_mix<C>(w, st, n, L, 6, 7, t, st.dA0[L], nullptr, st.A1[L], st.dA1[L], nullptr, s);
}

template <int C>
fmd_status node_tc_sender(const GraphArgs& ga, const FusedWeights& w, const FusedState& st, int64_t n,
                          int group_grid, bool single, size_t node_smem, int L, cudaStream_t s) {
    const int eg = int((n * C + 255) / 256 < int64_t(kNumSMs) * 8 ? (n * C + 255) / 256 : int64_t(kNumSMs) * 8);
    const int Lp = L - 1;
    if (single) tcn_sender_gather_kernel<C, 1><<<group_grid, kQ * C, node_smem, s>>>(ga, w, st, L, st.A0[L], st.A1[L]);
    else tcn_sender_gather_kernel<C, kG><<<group_grid, kQ * C, node_smem, s>>>(ga, w, st, L, st.A0[L], st.A1[L]);
    fmd_status r = check_launch();
    if (r != FMD_OK) return r;
    r = node_mix<C>(w, st, n, L, 10, 11, st.A0[L], st.s_t[L], nullptr, st.A1[L], st.v_t[L], nullptr, s);
    if (r != FMD_OK) return r;
    tcn_sender_mid_kernel<C><<<eg, 256, 0, s>>>(w, st, L, st.s_t[L], st.v_t[L], n);
    if ((r = check_launch()) != FMD_OK) return r;
    r = node_mix<C>(w, st, n, Lp, 8, 9, st.s_t[L], st.s_out[Lp], nullptr, st.v_t[L], st.v_out[Lp], nullptr, s);
    if (r != FMD_OK) return r;
    tcn_sender_prod_kernel<C><<<eg, 256, 0, s>>>(w, st, Lp, st.s_out[Lp], st.v_out[Lp], n);
    if ((r = check_launch()) != FMD_OK) return r;
    return node_mix<C>(w, st, n, Lp, 6, 7, st.s_out[Lp], st.dA0[Lp], nullptr, st.v_out[Lp], st.dA1[Lp], nullptr, s);
}

template <int C>
fmd_status launch_step(const EdgeArgs& ea, const GraphArgs& ga, const FusedWeights& w, const FusedState& st,
                       int64_t atoms_per_system, int32_t n_systems, float* forces, double* total, int32_t stages,
                       cudaStream_t s) {
    const auto on = [stages](int bit) { return (stages >> bit) & 1; };
    const int64_t n_tiles = (ea.n_edges + kTF - 1) / kTF;
    const int edge_grid = int(n_tiles < int64_t(kNumSMs) * 8 ? n_tiles : int64_t(kNumSMs) * 8);
    const int atom_grid = int(ga.n_atoms < int64_t(kNumSMs) * 16 ? ga.n_atoms : int64_t(kNumSMs) * 16);
    // the per-edge backward: a warp per receiver run once every SM has several CTAs of such warps
    const int bwd_per_warp = ga.n_atoms >= int64_t(kNumSMs) * 16 ? 1 : 0;
    const int msg_bwd_grid = bwd_per_warp ? int((ga.n_atoms + kMsgBwdWarps - 1) / kMsgBwdWarps) : atom_grid;
    // fewer groups than SMs: one CTA per entry of the group table (4x the CTAs, the same results)
    const bool single = st.n_groups < kNumSMs;
    const int64_t units = single ? st.n_groups * kG : st.n_groups;
    const int group_grid = int(units < int64_t(kNumSMs) * 16 ? units : int64_t(kNumSMs) * 16);
    const int64_t b_tiles = (ea.n_edges + kTB - 1) / kTB;
    const int bwd_grid = int(b_tiles < int64_t(kNumSMs) * 8 ? b_tiles : int64_t(kNumSMs) * 8);
    const size_t node_smem = sizeof(NodeSmem<C>);
    fmd_status stt;
    const size_t fwd_smem = sizeof(EdgeFwdSmem) + sizeof(float) * kH * 4 * C;  // + the staged W4^T
    if ((stt = grant_dynamic_smem((const void*)edge_fwd_kernel<C>, fwd_smem)) != FMD_OK) return stt;
    if ((stt = grant_dynamic_smem((const void*)edge_bwd_kernel<C>, sizeof(EdgeBwdSmem))) != FMD_OK) return stt;
    // the six node kernels (three, for 4 and 1 atoms per CTA) share one NodeSmem size: grant each once
    {
        const void* kernels[12] = {(const void*)node_fwd_kernel<C, kG>,    (const void*)node_fwd_kernel<C, 1>,
                                   (const void*)node_last_kernel<C, kG>,   (const void*)node_last_kernel<C, 1>,
                                   (const void*)sender_node_kernel<C, kG>, (const void*)sender_node_kernel<C, 1>,
                                   (const void*)tcn_last_pre_kernel<C, kG>, (const void*)tcn_last_pre_kernel<C, 1>,
                                   (const void*)tcn_last_post_kernel<C, kG>, (const void*)tcn_last_post_kernel<C, 1>,
                                   (const void*)tcn_sender_gather_kernel<C, kG>,
                                   (const void*)tcn_sender_gather_kernel<C, 1>};
        // the largest shared-memory carveout: two CTAs of a node kernel per SM
        for (const void* kernel : kernels)
            if ((stt = grant_dynamic_smem(kernel, node_smem, true)) != FMD_OK) return stt;
    }
    const int L = w.n_layers;
    const bool tc = use_radial_tc(w, st, ea.n_edges);
    const bool ntc = use_node_tc(w, tc);
    const int geom_grid = int((ea.n_edges + kTG - 1) / kTG < int64_t(kNumSMs) * 8 ? (ea.n_edges + kTG - 1) / kTG
                                                                                  : int64_t(kNumSMs) * 8);
    if (tc && n_tiles > 0 && on(0)) {
        edge_geom_tc_kernel<<<geom_grid, 256, 0, s>>>(ea, w, st);
        if ((stt = check_launch()) != FMD_OK) return stt;
        if ((stt = radial_tc_forward(w, st, ea.n_edges, C, s)) != FMD_OK) return stt;
    } else if (n_tiles > 0 && on(0)) {
        edge_fwd_kernel<C><<<edge_grid, 256, fwd_smem, s>>>(ea, w, st);
    }
    for (int l = 0; l < L; ++l) {
        if (on(1)) {
            if (l == 0) message_fused_kernel<C, 2><<<atom_grid, 32 * kMsgWarps, 0, s>>>(ga, w, st, l);
            else message_fused_kernel<C, 4><<<atom_grid, 32 * kMsgWarps, 0, s>>>(ga, w, st, l);
        }
        if (l < L - 1 && on(2)) {
            if (ntc) {
                if ((stt = check_launch()) != FMD_OK) return stt;
                if ((stt = node_tc_forward<C>(w, st, ga.n_atoms, group_grid, single, node_smem, l, s)) != FMD_OK)
                    return stt;
            } else if (single) node_fwd_kernel<C, 1><<<group_grid, kQ * C, node_smem, s>>>(w, st, l);
            else node_fwd_kernel<C, kG><<<group_grid, kQ * C, node_smem, s>>>(w, st, l);
        }
    }
    if (on(3)) {
        if (ntc) {
            if ((stt = check_launch()) != FMD_OK) return stt;
            if ((stt = node_tc_forward<C>(w, st, ga.n_atoms, group_grid, single, node_smem, L - 1, s)) != FMD_OK)
                return stt;
        } else if (single) node_last_kernel<C, 1><<<group_grid, kQ * C, node_smem, s>>>(w, st, L - 1);
        else node_last_kernel<C, kG><<<group_grid, kQ * C, node_smem, s>>>(w, st, L - 1);
    }
    for (int l = L - 1; l >= 1; --l) {
        if (on(4)) msg_bwd_edge_kernel<C, 4><<<msg_bwd_grid, 32 * kMsgBwdWarps, 0, s>>>(ga, w, st, l, l != L - 1, bwd_per_warp);
        if (on(5)) {
            if (ntc) {
                if ((stt = check_launch()) != FMD_OK) return stt;
                if ((stt = node_tc_sender<C>(ga, w, st, ga.n_atoms, group_grid, single, node_smem, l, s)) != FMD_OK)
                    return stt;
            } else if (single) sender_node_kernel<C, 1><<<group_grid, kQ * C, node_smem, s>>>(ga, w, st, l);
            else sender_node_kernel<C, kG><<<group_grid, kQ * C, node_smem, s>>>(ga, w, st, l);
        }
    }
    if (on(4)) msg_bwd_edge_kernel<C, 2><<<msg_bwd_grid, 32 * kMsgBwdWarps, 0, s>>>(ga, w, st, 0, L != 1, bwd_per_warp);
    if (tc && b_tiles > 0 && on(6)) {
        if ((stt = check_launch()) != FMD_OK) return stt;
        if ((stt = radial_tc_backward(w, st, ea.n_edges, C, s)) != FMD_OK) return stt;
        edge_geom_bwd_tc_kernel<<<geom_grid, 256, 0, s>>>(ea, w, st);
    } else if (b_tiles > 0 && on(6)) {
        edge_bwd_kernel<C><<<bwd_grid, kBT, sizeof(EdgeBwdSmem), s>>>(ea, w, st);
    }
    if (on(7)) {
        int64_t chunks = (atoms_per_system + kForceWarps - 1) / kForceWarps;
        if (chunks > 64) chunks = 64;
        forces_kernel<<<dim3(unsigned(chunks), unsigned(n_systems)), 32 * kForceWarps, 0, s>>>(
            ga, st.g_r, st.node_energy, atoms_per_system, forces, total);
    }
    return check_launch();
}

}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_mace_fused_step(const fmd_mace_fused_weights* weights, const fmd_mace_fused_state* state,
                               const float* positions, const float* cell, const int32_t* edge_index,
                               const float* edge_image, int64_t n_edges, const int64_t* n_real_edges,
                               const int64_t* recv_off,
                               const int64_t* send_off, const int32_t* send_perm, int64_t atoms_per_system,
                               int32_t n_systems, int32_t channels, float* forces, double* energy, int32_t stages,
                               void* stream) {
    // the edge arrays may be NULL (empty tensors) when there are no edge rows: nothing reads them then
    if (weights == nullptr || state == nullptr || positions == nullptr || cell == nullptr ||
        (n_edges > 0 && (edge_index == nullptr || edge_image == nullptr || send_perm == nullptr)) ||
        recv_off == nullptr || send_off == nullptr || forces == nullptr || energy == nullptr || n_edges < 0 ||
        atoms_per_system < 1 || n_systems < 1)
        return FMD_ERR_INVALID_ARGUMENT;
    FusedWeights w{};
    FusedState st{};
    const fmd_mace_fused_weights& h = *weights;
    if (h.n_layers < 1 || h.n_layers > kMaxLayers || h.n_basis < 1 || h.n_basis > 16 || h.readout_hidden < 1 ||
        h.readout_hidden > 32 || h.radial_hidden != kH)
        return FMD_ERR_UNSUPPORTED;
    for (int l = 0; l < h.n_layers; ++l) {
        w.w1t[l] = h.radial_w1t[l]; w.w2t[l] = h.radial_w2t[l]; w.w3t[l] = h.radial_w3t[l]; w.w4t[l] = h.radial_w4t[l];
        w.w1[l] = h.radial_w1[l]; w.w2[l] = h.radial_w2[l]; w.w3[l] = h.radial_w3[l]; w.w4[l] = h.radial_w4[l];
        w.lin0[l] = h.lin0[l]; w.lin1[l] = h.lin1[l]; w.lin0t[l] = h.lin0t[l]; w.lin1t[l] = h.lin1t[l];
        w.out0[l] = h.out0[l]; w.out1[l] = h.out1[l]; w.out0t[l] = h.out0t[l]; w.out1t[l] = h.out1t[l];
        w.up0[l] = h.up0[l]; w.up1[l] = h.up1[l]; w.up0t[l] = h.up0t[l]; w.up1t[l] = h.up1t[l];
        w.prod0[l] = h.prod0[l]; w.prod1[l] = h.prod1[l];
        w.skip0[l] = h.skip0[l]; w.skip1[l] = h.skip1[l]; w.skip0t[l] = h.skip0t[l]; w.skip1t[l] = h.skip1t[l];
        st.R[l] = state->R[l]; st.dR[l] = state->dR[l]; st.s_t[l] = state->s_t[l]; st.v_t[l] = state->v_t[l];
        st.A0[l] = state->A0[l]; st.A1[l] = state->A1[l]; st.A0l[l] = state->A0l[l]; st.A1l[l] = state->A1l[l];
        st.s_out[l] = state->s_out[l]; st.v_out[l] = state->v_out[l]; st.dA0[l] = state->dA0[l];
        st.dA1[l] = state->dA1[l]; st.ds_skip[l] = state->ds_skip[l]; st.dv_skip[l] = state->dv_skip[l];
    }
    w.s_t0 = h.s_t0; w.r0 = h.r0; w.ra = h.ra; w.rb = h.rb; w.e0 = h.e0;
    w.scale = h.scale; w.shift = h.shift; w.n_layers = h.n_layers; w.n_basis = h.n_basis; w.poly_p = h.poly_p;
    w.readout_hidden = h.readout_hidden; w.r_max = h.r_max; w.inv_avg = h.inv_avg;
    w.tc_min_edges = h.radial_tc_min_edges;
    for (int m = 0; m < 12; ++m)
        for (int l = 0; l < h.n_layers; ++l) {
            w.ntc_hi[m][l] = h.node_tc_hi[m][l];
            w.ntc_lo[m][l] = h.node_tc_lo[m][l];
        }
    for (int d = 0; d < 2; ++d)
        for (int l = 0; l < h.n_layers; ++l) {
            w.skip_hi[d][l] = h.skip_tc_hi[d][l];
            w.skip_lo[d][l] = h.skip_tc_lo[d][l];
        }
    st.elem_order = state->elem_order;
    st.elem_rank = state->elem_rank;
    st.n_runs = state->n_elem_runs;
    st.runs_host = state->elem_runs_host;
    for (int k = 0; k < 3; ++k)
        for (int l = 0; l < h.n_layers; ++l) {
            w.tc_hi[k][l] = h.radial_tc_hi[k][l]; w.tc_lo[k][l] = h.radial_tc_lo[k][l];
            w.tc_t_hi[k][l] = h.radial_tc_t_hi[k][l]; w.tc_t_lo[k][l] = h.radial_tc_t_lo[k][l];
            st.pre[k][l] = state->radial_pre[k][l];
        }
    st.flags = state->flags;
    st.ysh = reinterpret_cast<float4*>(state->ysh); st.dY = state->dY; st.g_r = state->g_r;
    st.e_term0 = state->e_term0; st.node_energy = state->node_energy; st.elem = state->elem;
    st.groups = state->groups; st.n_groups = state->n_groups;
    if (!aligned16(state->ysh)) return FMD_ERR_INVALID_ARGUMENT;
    const EdgeArgs ea{positions, cell, edge_index, edge_image, n_edges, n_real_edges, channels};
    const GraphArgs ga{edge_index, recv_off, send_off, send_perm, atoms_per_system * n_systems};
    cudaStream_t s = as_stream(stream);
    switch (channels) {
        case 32: return launch_step<32>(ea, ga, w, st, atoms_per_system, n_systems, forces, energy, stages, s);
        case 64: return launch_step<64>(ea, ga, w, st, atoms_per_system, n_systems, forces, energy, stages, s);
        case 128: return launch_step<128>(ea, ga, w, st, atoms_per_system, n_systems, forces, energy, stages, s);
        default: return FMD_ERR_UNSUPPORTED;
    }
}

}  // extern "C"
