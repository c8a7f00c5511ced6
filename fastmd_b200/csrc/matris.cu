// MatRIS geometry, radial and three-body bases, and the explicit force /
// virial reduction of the MatRIS potential.
//
// The model's energy depends on positions only through the directed edge
// vectors v_e = x[centre] - (x[neighbour] + image_e @ L): through the bond
// lengths d[u2d[u]] (the Bessel bases of every bond) and through the unit
// vectors u_e = v_e / d_e of the triplets' two edges (the angle). The model
// is differentiated (by autograd over this library's kernels) with respect
// to those two leaves only; this file turns their gradients into dE/dv_e,
// then into forces F = -dE/dx and the virial W = sum_e v_e (x) dE/dv_e, with
// per-atom CSR sums (no atomics: the results do not depend on the launch).
//
// Kernels:
//   matris_geometry_kernel   one thread per directed edge: d_e, u_e
//   bessel_kernel / _bwd     one thread per (bond, basis function) / per bond
//   threebody_kernel / _bwd  one thread per triplet (basis, dE/dcos), then one
//                            warp per bond folding its triplets into dE/du of
//                            its two directed rows
//   forces_kernel            one warp per atom over its centre and neighbour
//                            edges (forces, the atom's virial row)
//   virial_reduce_kernel     one CTA: the per-atom virial rows in FP64, in a
//                            fixed order, symmetrised and scaled.

#include <math.h>

#include "common.cuh"

namespace fmd {

namespace {

constexpr int kThreads = 256;

__global__ void matris_geometry_kernel(const float* __restrict__ positions, const float* __restrict__ cell,
                                       const int32_t* __restrict__ edge_index, const float* __restrict__ edge_image,
                                       int64_t n_edges, int64_t n_atoms, float* __restrict__ length,
                                       float* __restrict__ unit, int32_t* flags) {
    __shared__ float L[9];
    if (threadIdx.x < 9) L[threadIdx.x] = cell[threadIdx.x];
    __syncthreads();
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges;
         e += int64_t(gridDim.x) * blockDim.x) {
        int64_t c = edge_index[2 * e], n = edge_index[2 * e + 1];
        if (c < 0 || c >= n_atoms || n < 0 || n >= n_atoms) {
            raise_flag(flags, FMD_FLAG_INDEX_RANGE);
            c = 0;
            n = 0;
        }
        const float i0 = edge_image[3 * e], i1 = edge_image[3 * e + 1], i2 = edge_image[3 * e + 2];
        float v[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            // image @ L summed over the three lattice rows in order, then centre - (neighbour + shift)
            const float shift = (i0 * L[j] + i1 * L[3 + j]) + i2 * L[6 + j];
            v[j] = positions[3 * c + j] - (positions[3 * n + j] + shift);
        }
        const float d = sqrtf((v[0] * v[0] + v[1] * v[1]) + v[2] * v[2]);
        length[e] = d;
        unit[3 * e] = v[0] / d;
        unit[3 * e + 1] = v[1] / d;
        unit[3 * e + 2] = v[2] / d;
    }
}

struct BesselArgs {
    const float* length;
    const int32_t* u2d;
    int64_t n_bonds;
    int64_t n_edges;
    const float* freq[2];
    float cutoff[2];
    float exponent;
    int32_t n_basis;
};

__device__ __forceinline__ float envelope(float x, float p, float a, float b, float c) {
    return x < 1.f ? 1.f + a * powf(x, p) + b * powf(x, p + 1.f) + c * powf(x, p + 2.f) : 0.f;
}

__device__ __forceinline__ float envelope_grad(float x, float p, float a, float b, float c) {
    // d env / d x
    return x < 1.f ? a * p * powf(x, p - 1.f) + b * (p + 1.f) * powf(x, p) + c * (p + 2.f) * powf(x, p + 1.f) : 0.f;
}

// the bond's length: length[u2d[u]] (u2d null: length[u], one entry per bond)
__device__ __forceinline__ float bond_length(const BesselArgs& a, int64_t u) {
    int64_t e = a.u2d != nullptr ? int64_t(a.u2d[u]) : u;
    if (e < 0 || e >= a.n_edges) e = 0;
    return a.length[e];
}

// rbf_s[u, k] = env(d / rc_s) * sqrt(2 / rc_s) * sin(f_sk * d * (1 / rc_s)) / d for k < n_basis, 0 up to ldr
__global__ void bessel_kernel(BesselArgs a, float* __restrict__ rbf_atom, float* __restrict__ rbf_line,
                              int64_t ldr) {
    const int64_t total = a.n_bonds * 2 * ldr;
    const float p = a.exponent;
    const float ca = -(p + 1.f) * (p + 2.f) / 2.f, cb = p * (p + 2.f), cc = -p * (p + 1.f) / 2.f;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t u = i / (2 * ldr);
        const int col = int(i - u * 2 * ldr);
        const int s = col >= ldr ? 1 : 0, k = col - s * int(ldr);
        float value = 0.f;
        if (k < a.n_basis) {
            const float d = bond_length(a, u);
            const float rc = a.cutoff[s];
            const float norm = sqrtf(2.f * (1.f / rc));
            const float basis = norm * sinf(a.freq[s][k] * (d * (1.f / rc))) / d;
            value = envelope(d / rc, p, ca, cb, cc) * basis;
        }
        (s == 0 ? rbf_atom : rbf_line)[u * ldr + k] = value;
    }
}

__global__ void bessel_bwd_kernel(BesselArgs a, const float* __restrict__ grad_atom,
                                  const float* __restrict__ grad_line, int64_t ldg,
                                  float* __restrict__ grad_length) {
    const float p = a.exponent;
    const float ca = -(p + 1.f) * (p + 2.f) / 2.f, cb = p * (p + 2.f), cc = -p * (p + 1.f) / 2.f;
    for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < a.n_bonds;
         u += int64_t(gridDim.x) * blockDim.x) {
        const float d = bond_length(a, u);
        float acc = 0.f;
        for (int s = 0; s < 2; ++s) {
            const float rc = a.cutoff[s], inv = 1.f / rc;
            const float norm = sqrtf(2.f * inv);
            const float x = d / rc;
            const float env = envelope(x, p, ca, cb, cc), denv = envelope_grad(x, p, ca, cb, cc) * inv;
            for (int k = 0; k < a.n_basis; ++k) {
                const float f = a.freq[s][k];
                float sn, cs;
                sincosf(f * (d * inv), &sn, &cs);
                const float basis = norm * sn / d;
                const float dbasis = norm * (f * inv * cs / d - sn / (d * d));
                acc += (s == 0 ? grad_atom : grad_line)[u * ldg + k] * (denv * basis + env * dbasis);
            }
        }
        grad_length[u] = acc;
    }
}

struct TripletArgs {
    const float* unit;
    const int32_t* line_graph;  // [T, 5] (atom, u1, e1, u2, e2)
    int64_t n_triplets;
    int64_t n_edges;
    const float* freq;
    int32_t n_freq;
};

constexpr float kAngleShrink = 1.f - 1e-6f;  // cos scaled into acos's open domain (feature_embed.py:441)

__device__ __forceinline__ float triplet_cos(const TripletArgs& a, int64_t t, int64_t* e1_out, int64_t* e2_out) {
    int64_t e1 = a.line_graph[5 * t + 2], e2 = a.line_graph[5 * t + 4];
    if (e1 < 0 || e1 >= a.n_edges) e1 = 0;
    if (e2 < 0 || e2 >= a.n_edges) e2 = 0;
    *e1_out = e1;
    *e2_out = e2;
    const float* p = a.unit + 3 * e1;
    const float* q = a.unit + 3 * e2;
    return ((p[0] * q[0] + p[1] * q[1]) + p[2] * q[2]) * kAngleShrink;
}

// basis[t] = [2^-1/2, sin(f_k theta)..., cos(f_k theta)...] / sqrt(pi), theta = acos(cos)
__global__ void threebody_kernel(TripletArgs a, float* __restrict__ basis, int64_t ldb, int32_t* flags) {
    const float inv_scale = 1.f / sqrtf(3.14159265358979323846f);
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < a.n_triplets;
         t += int64_t(gridDim.x) * blockDim.x) {
        int64_t e1, e2;
        const int64_t r1 = a.line_graph[5 * t + 2], r2 = a.line_graph[5 * t + 4];
        if (r1 < 0 || r1 >= a.n_edges || r2 < 0 || r2 >= a.n_edges) raise_flag(flags, FMD_FLAG_INDEX_RANGE);
        const float theta = acosf(triplet_cos(a, t, &e1, &e2));
        float* out = basis + t * ldb;
        out[0] = 0.70710678118654752f * inv_scale;
        for (int k = 0; k < a.n_freq; ++k) {
            float sn, cs;
            sincosf(theta * a.freq[k], &sn, &cs);
            out[1 + k] = sn * inv_scale;
            out[1 + a.n_freq + k] = cs * inv_scale;
        }
        for (int64_t k = 1 + 2 * a.n_freq; k < ldb; ++k) out[k] = 0.f;  // the row's padding
    }
}

// dE/dc of every triplet, c = u1 . u2 the raw cosine: sum_k g_k dbasis_k/dtheta * dtheta/dcos' * s for
// cos' = s c (s = 1 - 1e-6), with
// 1 - cos'^2 = |u1 x u2|^2 + c^2 (1 - s^2) (no cancellation near 0 and pi)
__global__ void threebody_grad_cos_kernel(TripletArgs a, const float* __restrict__ grad_basis, int64_t ldg,
                                          float* __restrict__ grad_cos) {
    const float inv_scale = 1.f / sqrtf(3.14159265358979323846f);
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < a.n_triplets;
         t += int64_t(gridDim.x) * blockDim.x) {
        int64_t e1, e2;
        const float c = triplet_cos(a, t, &e1, &e2);
        const float theta = acosf(c);
        const float* g = grad_basis + t * ldg;
        float dtheta = 0.f;
        for (int k = 0; k < a.n_freq; ++k) {
            const float f = a.freq[k];
            float sn, cs;
            sincosf(theta * f, &sn, &cs);
            dtheta += (g[1 + k] * cs - g[1 + a.n_freq + k] * sn) * f;
        }
        const float* p = a.unit + 3 * e1;
        const float* q = a.unit + 3 * e2;
        const float x0 = p[1] * q[2] - p[2] * q[1], x1 = p[2] * q[0] - p[0] * q[2], x2 = p[0] * q[1] - p[1] * q[0];
        const float raw = c / kAngleShrink;
        const float sin2 = (x0 * x0 + x1 * x1 + x2 * x2) + raw * raw * (1.f - kAngleShrink * kAngleShrink);
        grad_cos[t] = -dtheta * inv_scale * kAngleShrink * rsqrtf(fmaxf(sin2, 1e-30f));
    }
}

// dE/du for the two directed rows (pair[u, 0], pair[u, 1]) of every bond u: the triplets whose first
// bond is u (CSR perm1/off1) add g_t u[e2] to their e1 row, those whose second bond is u (perm2/off2)
// add g_t u[e1] to their e2 row; each row summed in CSR order by one lane group.
__global__ void threebody_fold_kernel(TripletArgs a, const float* __restrict__ grad_cos,
                                      const int64_t* __restrict__ pair_index, int64_t n_bonds,
                                      const int64_t* __restrict__ perm1, const int64_t* __restrict__ off1,
                                      const int64_t* __restrict__ perm2, const int64_t* __restrict__ off2,
                                      float* __restrict__ grad_unit) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t u = warp; u < n_bonds; u += n_warps) {
        const int64_t rows[2] = {pair_index[2 * u], pair_index[2 * u + 1]};
        float acc[2][3] = {{0.f, 0.f, 0.f}, {0.f, 0.f, 0.f}};
        for (int side = 0; side < 2; ++side) {
            const int64_t* perm = side == 0 ? perm1 : perm2;
            const int64_t* off = side == 0 ? off1 : off2;
            const int64_t lo = off[u], hi = off[u + 1];
            for (int64_t i = lo + lane; i < hi; i += 32) {
                const int64_t t = perm[i];
                const int64_t own = a.line_graph[5 * t + (side == 0 ? 2 : 4)];
                const int64_t other = a.line_graph[5 * t + (side == 0 ? 4 : 2)];
                if (other < 0 || other >= a.n_edges) continue;
                const float g = grad_cos[t];
                const int slot = own == rows[0] ? 0 : 1;
                const float* q = a.unit + 3 * other;
                acc[slot][0] += g * q[0];
                acc[slot][1] += g * q[1];
                acc[slot][2] += g * q[2];
            }
        }
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int j = 0; j < 3; ++j)
#pragma unroll
                for (int m = 16; m > 0; m >>= 1) acc[s][j] += __shfl_xor_sync(0xffffffffu, acc[s][j], m);
        if (lane < 6) {
            const int s = lane / 3, j = lane % 3;
            const int64_t row = rows[s];
            if (row >= 0 && row < a.n_edges) grad_unit[3 * row + j] = acc[s][j];
        }
    }
}

// env[t, :] = base[u2[t], :] * base[u1[t], :] (the source bond's envelope times the target bond's), float4
// columns; width % 4 == 0, rows 16-byte aligned
__global__ void line_envelope_kernel(const float* __restrict__ base, int64_t ldb, const int32_t* __restrict__ lg,
                                     int64_t n_triplets, int64_t n_bonds, int width, float* __restrict__ env,
                                     int64_t lde, int32_t* flags) {
    const int wv = width / 4;
    const int64_t total = n_triplets * wv;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t t = i / wv;
        const int c = int(i - t * wv);
        int64_t u1 = lg[5 * t + 1], u2 = lg[5 * t + 3];
        if (u1 < 0 || u1 >= n_bonds || u2 < 0 || u2 >= n_bonds) {
            raise_flag(flags, FMD_FLAG_INDEX_RANGE);
            u1 = 0;
            u2 = 0;
        }
        st4(env + t * lde + 4 * c, f4_mul(ldg4(base + u2 * ldb + 4 * c), ldg4(base + u1 * ldb + 4 * c)));
    }
}

// grad_base[u] = sum over the triplets whose target bond is u (CSR perm1/off1) of g[t] * base[u2[t]], plus
// over those whose source bond is u (perm2/off2) of g[t] * base[u1[t]]: a CTA of kEnvWarps warps per
// (bond, 128 columns), warp w taking every kEnvWarps-th triplet of each side (two triplets' loads in flight),
// the warp partials added in warp order (deterministic, no atomics)
constexpr int kEnvWarps = 8;

__global__ void __launch_bounds__(32 * kEnvWarps) line_envelope_bwd_kernel(
    const float* __restrict__ base, int64_t ldb, const int32_t* __restrict__ lg, int64_t n_bonds, int width,
    const float* __restrict__ grad, int64_t ldg, const int64_t* __restrict__ perm1, const int64_t* __restrict__ off1,
    const int64_t* __restrict__ perm2, const int64_t* __restrict__ off2, float* __restrict__ grad_base, int64_t ldo) {
    __shared__ float4 part[kEnvWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunks = (width / 4 + 31) / 32;
    for (int64_t task = blockIdx.x; task < n_bonds * chunks; task += gridDim.x) {
        const int64_t u = task / chunks;
        const int v = int(task - u * chunks) * 32 + lane;
        const bool col_ok = v < width / 4;
        float4 acc = f4_zero();
        for (int side = 0; side < 2; ++side) {
            const int64_t* perm = side == 0 ? perm1 : perm2;
            const int64_t* off = side == 0 ? off1 : off2;
            const int col = side == 0 ? 3 : 1;
            const int64_t end = off[u + 1];
            int64_t j = off[u] + warp;
            for (; j + kEnvWarps < end; j += 2 * kEnvWarps) {
                const int64_t t0 = perm[j], t1 = perm[j + kEnvWarps];
                int64_t o0 = lg[5 * t0 + col], o1 = lg[5 * t1 + col];
                if (o0 < 0 || o0 >= n_bonds) o0 = 0;
                if (o1 < 0 || o1 >= n_bonds) o1 = 0;
                if (col_ok) {
                    const float4 x0 = ldg4(grad + t0 * ldg + 4 * v), y0 = ldg4(base + o0 * ldb + 4 * v);
                    const float4 x1 = ldg4(grad + t1 * ldg + 4 * v), y1 = ldg4(base + o1 * ldb + 4 * v);
                    acc = f4_add(acc, f4_mul(x0, y0));
                    acc = f4_add(acc, f4_mul(x1, y1));
                }
            }
            for (; j < end; j += kEnvWarps) {
                const int64_t t = perm[j];
                int64_t o = lg[5 * t + col];
                if (o < 0 || o >= n_bonds) o = 0;
                if (col_ok) acc = f4_add(acc, f4_mul(ldg4(grad + t * ldg + 4 * v), ldg4(base + o * ldb + 4 * v)));
            }
        }
        part[warp][lane] = acc;
        __syncthreads();
        if (warp == 0 && col_ok) {
            float4 total = part[0][lane];
#pragma unroll
            for (int w = 1; w < kEnvWarps; ++w) total = f4_add(total, part[w][lane]);
            st4(grad_base + u * ldo + 4 * v, total);
        }
        __syncthreads();
    }
}

struct ForceArgs {
    const float* length;
    const float* unit;
    const float* grad_length;  // [U] per bond, or null
    const float* grad_unit;    // [E, 3], or null
    const int32_t* d2u;
    const int32_t* u2d;
    const int32_t* edge_index;
    int64_t n_edges;
    int64_t n_bonds;
    int64_t n_atoms;
    const int64_t* recv_perm;  // null: identity (edges sorted by centre)
    const int64_t* recv_off;
    const int64_t* send_perm;
    const int64_t* send_off;
};

// dE/dv_e = g_d u + (g_u - (g_u . u) u) / d, g_d the bond length gradient on the bond's stored direction
__device__ __forceinline__ void edge_grad(const ForceArgs& a, int64_t e, float g[3]) {
    float gd = 0.f;
    if (a.grad_length != nullptr) {
        const int64_t u = a.d2u[e];
        if (u >= 0 && u < a.n_bonds && a.u2d[u] == e) gd = a.grad_length[u];
    }
    const float* uv = a.unit + 3 * e;
    float gu[3] = {0.f, 0.f, 0.f};
    if (a.grad_unit != nullptr) {
        gu[0] = a.grad_unit[3 * e];
        gu[1] = a.grad_unit[3 * e + 1];
        gu[2] = a.grad_unit[3 * e + 2];
    }
    const float dot = (gu[0] * uv[0] + gu[1] * uv[1]) + gu[2] * uv[2];
    const float inv_d = 1.f / a.length[e];
#pragma unroll
    for (int j = 0; j < 3; ++j) g[j] = gd * uv[j] + (gu[j] - dot * uv[j]) * inv_d;
}

// forces[i] = sum_{e: neighbour i} g_e - sum_{e: centre i} g_e; virial_rows[i] = sum_{e: centre i} v_e (x) g_e
__global__ void forces_kernel(ForceArgs a, float* __restrict__ forces, double* __restrict__ virial_rows) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t i = warp; i < a.n_atoms; i += n_warps) {
        float f[3] = {0.f, 0.f, 0.f};
        double w[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
        for (int64_t k = a.recv_off[i] + lane; k < a.recv_off[i + 1]; k += 32) {
            const int64_t e = a.recv_perm != nullptr ? a.recv_perm[k] : k;
            float g[3];
            edge_grad(a, e, g);
            const float d = a.length[e];
            const float* uv = a.unit + 3 * e;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                f[j] -= g[j];
#pragma unroll
                for (int m = 0; m < 3; ++m) w[3 * j + m] += double(uv[j] * d) * double(g[m]);
            }
        }
        for (int64_t k = a.send_off[i] + lane; k < a.send_off[i + 1]; k += 32) {
            float g[3];
            edge_grad(a, a.send_perm[k], g);
#pragma unroll
            for (int j = 0; j < 3; ++j) f[j] += g[j];
        }
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) {
#pragma unroll
            for (int j = 0; j < 3; ++j) f[j] += __shfl_xor_sync(0xffffffffu, f[j], m);
#pragma unroll
            for (int j = 0; j < 9; ++j) w[j] += __shfl_xor_sync(0xffffffffu, w[j], m);
        }
        if (lane < 3) forces[3 * i + lane] = f[lane];
        if (virial_rows != nullptr && lane < 9) virial_rows[9 * i + lane] = w[lane];
    }
}

// stress[j][m] = unit / |det L| * (W[j][m] + W[m][j]) / 2, W summed over the atoms in a fixed order in FP64
__global__ void virial_reduce_kernel(const double* __restrict__ rows, int64_t n_atoms, const float* __restrict__ cell,
                                     double unit, float* __restrict__ stress, double* __restrict__ virial) {
    __shared__ double part[kThreads][9];
    double acc[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = threadIdx.x; i < n_atoms; i += blockDim.x)
#pragma unroll
        for (int j = 0; j < 9; ++j) acc[j] += rows[9 * i + j];
#pragma unroll
    for (int j = 0; j < 9; ++j) part[threadIdx.x][j] = acc[j];
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s)
#pragma unroll
            for (int j = 0; j < 9; ++j) part[threadIdx.x][j] += part[threadIdx.x + s][j];
        __syncthreads();
    }
    if (threadIdx.x < 9) {
        const double L[9] = {cell[0], cell[1], cell[2], cell[3], cell[4], cell[5], cell[6], cell[7], cell[8]};
        const double det = L[0] * (L[4] * L[8] - L[5] * L[7]) - L[1] * (L[3] * L[8] - L[5] * L[6]) +
                           L[2] * (L[3] * L[7] - L[4] * L[6]);
        const double scale = unit / fabs(det);
        const int j = threadIdx.x / 3, m = threadIdx.x % 3;
        const double wjm = part[0][3 * j + m], wmj = part[0][3 * m + j];
        if (virial != nullptr) virial[threadIdx.x] = wjm;
        if (stress != nullptr) stress[threadIdx.x] = float(0.5 * (wjm + wmj) * scale);
    }
}

}  // namespace

}  // namespace fmd

using namespace fmd;

fmd_status fmd_matris_geometry(const float* positions, const float* cell, const int32_t* edge_index,
                               const float* edge_image, int64_t n_edges, int64_t n_atoms, float* length, float* unit,
                               int32_t* flags, void* stream) {
    if (n_edges < 0 || n_atoms < 1) return FMD_ERR_INVALID_ARGUMENT;
    if (n_edges == 0) return FMD_OK;
    if (positions == nullptr || cell == nullptr || edge_index == nullptr || edge_image == nullptr ||
        length == nullptr || unit == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    matris_geometry_kernel<<<grid_for(n_edges, kThreads), kThreads, 0, as_stream(stream)>>>(
        positions, cell, edge_index, edge_image, n_edges, n_atoms, length, unit, flags);
    return check_launch();
}

static fmd_status bessel_args(BesselArgs& a, const float* length, const int32_t* u2d, int64_t n_bonds,
                              int64_t n_edges, const float* freq_atom, const float* freq_line, int32_t n_basis,
                              float cutoff_atom, float cutoff_line, float exponent) {
    if (n_bonds < 0 || n_edges < 0 || n_basis < 1 || n_basis > 64 || !(cutoff_atom > 0.f) || !(cutoff_line > 0.f) ||
        !(exponent > 0.f))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_bonds > 0 && (length == nullptr || freq_atom == nullptr || freq_line == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    a = BesselArgs{length, u2d, n_bonds, n_edges, {freq_atom, freq_line}, {cutoff_atom, cutoff_line}, exponent,
                   n_basis};
    return FMD_OK;
}

fmd_status fmd_matris_bessel(const float* length, const int32_t* u2d, int64_t n_bonds, int64_t n_edges,
                             const float* freq_atom, const float* freq_line, int32_t n_basis, float cutoff_atom,
                             float cutoff_line, float exponent, float* rbf_atom, float* rbf_line, int64_t ldr,
                             void* stream) {
    BesselArgs a;
    fmd_status st = bessel_args(a, length, u2d, n_bonds, n_edges, freq_atom, freq_line, n_basis, cutoff_atom,
                                cutoff_line, exponent);
    if (st != FMD_OK) return st;
    if (n_bonds == 0) return FMD_OK;
    if (rbf_atom == nullptr || rbf_line == nullptr || ldr < n_basis) return FMD_ERR_INVALID_ARGUMENT;
    bessel_kernel<<<grid_for(n_bonds * 2 * ldr, kThreads), kThreads, 0, as_stream(stream)>>>(a, rbf_atom, rbf_line,
                                                                                             ldr);
    return check_launch();
}

fmd_status fmd_matris_bessel_bwd(const float* length, const int32_t* u2d, int64_t n_bonds, int64_t n_edges,
                                 const float* freq_atom, const float* freq_line, int32_t n_basis, float cutoff_atom,
                                 float cutoff_line, float exponent, const float* grad_atom, const float* grad_line,
                                 int64_t ldg, float* grad_length, void* stream) {
    BesselArgs a;
    fmd_status st = bessel_args(a, length, u2d, n_bonds, n_edges, freq_atom, freq_line, n_basis, cutoff_atom,
                                cutoff_line, exponent);
    if (st != FMD_OK) return st;
    if (n_bonds == 0) return FMD_OK;
    if (grad_atom == nullptr || grad_line == nullptr || grad_length == nullptr || ldg < n_basis)
        return FMD_ERR_INVALID_ARGUMENT;
    bessel_bwd_kernel<<<grid_for(n_bonds, kThreads), kThreads, 0, as_stream(stream)>>>(a, grad_atom, grad_line, ldg,
                                                                                        grad_length);
    return check_launch();
}

fmd_status fmd_matris_threebody(const float* unit, const int32_t* line_graph, int64_t n_triplets, int64_t n_edges,
                                const float* freq, int32_t n_freq, float* basis, int64_t ldb, int32_t* flags,
                                void* stream) {
    if (n_triplets < 0 || n_edges < 1 || n_freq < 1 || n_freq > 32) return FMD_ERR_INVALID_ARGUMENT;
    if (n_triplets == 0) return FMD_OK;
    if (unit == nullptr || line_graph == nullptr || freq == nullptr || basis == nullptr || ldb < 1 + 2 * n_freq)
        return FMD_ERR_INVALID_ARGUMENT;
    const TripletArgs a{unit, line_graph, n_triplets, n_edges, freq, n_freq};
    threebody_kernel<<<grid_for(n_triplets, kThreads), kThreads, 0, as_stream(stream)>>>(a, basis, ldb, flags);
    return check_launch();
}

fmd_status fmd_matris_threebody_bwd(const float* unit, const int32_t* line_graph, int64_t n_triplets,
                                    int64_t n_edges, const float* freq, int32_t n_freq, const float* grad_basis,
                                    int64_t ldg, const int64_t* pair_index, int64_t n_bonds, const int64_t* perm1,
                                    const int64_t* off1, const int64_t* perm2, const int64_t* off2, float* grad_cos,
                                    float* grad_unit, void* stream) {
    if (n_triplets < 0 || n_edges < 1 || n_bonds < 0 || n_freq < 1 || n_freq > 32 || 2 * n_bonds > n_edges)
        return FMD_ERR_INVALID_ARGUMENT;
    if (unit == nullptr || grad_unit == nullptr || pair_index == nullptr || off1 == nullptr || off2 == nullptr ||
        (n_triplets > 0 && (line_graph == nullptr || freq == nullptr || grad_basis == nullptr || grad_cos == nullptr ||
                            perm1 == nullptr || perm2 == nullptr || ldg < 1 + 2 * n_freq)))
        return FMD_ERR_INVALID_ARGUMENT;
    const cudaStream_t s = as_stream(stream);
    const TripletArgs a{unit, line_graph, n_triplets, n_edges, freq, n_freq};
    if (n_triplets > 0) {
        threebody_grad_cos_kernel<<<grid_for(n_triplets, kThreads), kThreads, 0, s>>>(a, grad_basis, ldg, grad_cos);
        fmd_status st = check_launch();
        if (st != FMD_OK) return st;
    }
    if (n_bonds == 0) return FMD_OK;
    threebody_fold_kernel<<<grid_for(n_bonds * 32, kThreads), kThreads, 0, s>>>(a, grad_cos, pair_index, n_bonds,
                                                                                 perm1, off1, perm2, off2, grad_unit);
    return check_launch();
}

static bool rows16(const float* p, int64_t ld) { return aligned16(p) && ld % 4 == 0; }

fmd_status fmd_matris_line_envelope(const float* base, int64_t ldb, const int32_t* line_graph, int64_t n_triplets,
                                    int64_t n_bonds, int32_t width, float* env, int64_t lde, int32_t* flags,
                                    void* stream) {
    if (n_triplets < 0 || n_bonds < 1 || width < 4 || width % 4 || ldb < width || lde < width)
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_triplets == 0) return FMD_OK;
    if (base == nullptr || line_graph == nullptr || env == nullptr) return FMD_ERR_INVALID_ARGUMENT;
    if (!rows16(base, ldb) || !rows16(env, lde)) return FMD_ERR_UNSUPPORTED;
    line_envelope_kernel<<<grid_for(n_triplets * (width / 4), kThreads), kThreads, 0, as_stream(stream)>>>(
        base, ldb, line_graph, n_triplets, n_bonds, width, env, lde, flags);
    return check_launch();
}

fmd_status fmd_matris_line_envelope_bwd(const float* base, int64_t ldb, const int32_t* line_graph, int64_t n_bonds,
                                        int32_t width, const float* grad, int64_t ldg, const int64_t* perm1,
                                        const int64_t* off1, const int64_t* perm2, const int64_t* off2,
                                        float* grad_base, int64_t ldo, void* stream) {
    if (n_bonds < 0 || width < 4 || width % 4 || ldb < width || ldg < width || ldo < width)
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_bonds == 0) return FMD_OK;
    if (base == nullptr || line_graph == nullptr || grad == nullptr || off1 == nullptr || off2 == nullptr ||
        grad_base == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    if (!rows16(base, ldb) || !rows16(grad, ldg) || !rows16(grad_base, ldo)) return FMD_ERR_UNSUPPORTED;
    const int64_t tasks = n_bonds * ((width / 4 + 31) / 32);
    const int grid = int(tasks < int64_t(kNumSMs) * 8 ? tasks : int64_t(kNumSMs) * 8);
    line_envelope_bwd_kernel<<<grid, 32 * kEnvWarps, 0, as_stream(stream)>>>(
        base, ldb, line_graph, n_bonds, width, grad, ldg, perm1, off1, perm2, off2, grad_base, ldo);
    return check_launch();
}

fmd_status fmd_matris_forces(const float* length, const float* unit, const float* grad_length,
                             const float* grad_unit, const int32_t* d2u, const int32_t* u2d,
                             const int32_t* edge_index, int64_t n_edges, int64_t n_bonds, int64_t n_atoms,
                             const int64_t* recv_perm, const int64_t* recv_off, const int64_t* send_perm,
                             const int64_t* send_off, const float* cell, double stress_unit, float* forces,
                             double* virial_rows, float* stress, double* virial, void* stream) {
    if (n_edges < 0 || n_bonds < 0 || n_atoms < 1) return FMD_ERR_INVALID_ARGUMENT;
    if (length == nullptr || unit == nullptr || d2u == nullptr || u2d == nullptr || edge_index == nullptr ||
        recv_off == nullptr || send_perm == nullptr || send_off == nullptr || forces == nullptr)
        return FMD_ERR_INVALID_ARGUMENT;
    if ((stress != nullptr || virial != nullptr) && (virial_rows == nullptr || cell == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    const cudaStream_t s = as_stream(stream);
    const ForceArgs a{length, unit, grad_length, grad_unit, d2u, u2d, edge_index, n_edges, n_bonds, n_atoms,
                      recv_perm, recv_off, send_perm, send_off};
    forces_kernel<<<grid_for(n_atoms * 32, kThreads), kThreads, 0, s>>>(a, forces, virial_rows);
    fmd_status st = check_launch();
    if (st != FMD_OK || (stress == nullptr && virial == nullptr)) return st;
    virial_reduce_kernel<<<1, kThreads, 0, s>>>(virial_rows, n_atoms, cell, stress_unit, stress, virial);
    return check_launch();
}
