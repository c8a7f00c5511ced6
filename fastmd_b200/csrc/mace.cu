// Kernels of the MACE-architecture message-passing potential (channels C,
// hidden irreps C x 0e + C x 1o, spherical harmonics l <= 1, correlation 3,
// Bessel radial basis with a polynomial cutoff), forward and the explicit
// backward that gives the forces dE/dr.
//
// Layouts: scalars s [N, C]; vectors v [N, 3, C] (component-major per atom,
// i.e. [3N, C] rows for the channel-mixing GEMMs); per-edge radial weights
// R [E, P*C] path-major (path p of channel k at p*C + k); edge geometry
// ysh [E, 4] = (sqrt(3) u, d) and the radial features phi [E, NB].
//
// The message kernels are the fused form of the hot path's gather ->
// per-edge product -> receiver-sorted segment sum: one CTA per receiver,
// one thread per channel, walking the receiver's CSR run in order (no
// atomics, no [E, C] intermediate in HBM); the backward walks the same run
// for the per-edge gradients and the sender CSR for the gathered rows.

#include "common.cuh"

namespace fmd {

constexpr float kSqrt3 = 1.7320508075688772f;
constexpr float kInvSqrt3 = 0.5773502691896258f;
constexpr int kMaxBasis = 16;

struct Geo {
    float r_max;
    int n_basis;
    int p;          // polynomial cutoff exponent
};

__device__ __forceinline__ float3 edge_vector(const float* pos, const float* cell, const int32_t* edge_index,
                                              const float* edge_image, int64_t e) {
    const int64_t i = edge_index[2 * e], j = edge_index[2 * e + 1];
    const float ix = edge_image[3 * e], iy = edge_image[3 * e + 1], iz = edge_image[3 * e + 2];
    // shift = image @ cell, row by row (no GEMM)
    const float sx = (ix * cell[0] + iy * cell[3]) + iz * cell[6];
    const float sy = (ix * cell[1] + iy * cell[4]) + iz * cell[7];
    const float sz = (ix * cell[2] + iy * cell[5]) + iz * cell[8];
    return make_float3((pos[3 * j] - pos[3 * i]) + sx, (pos[3 * j + 1] - pos[3 * i + 1]) + sy,
                       (pos[3 * j + 2] - pos[3 * i + 2]) + sz);
}

// polynomial cutoff f(x) = 1 - (p+1)(p+2)/2 x^p + p(p+2) x^(p+1) - p(p+1)/2 x^(p+2), x < 1
__device__ __forceinline__ void poly_cutoff(float d, const Geo& g, float& f, float& df) {
    const float x = d / g.r_max;
    if (!(x < 1.0f)) {
        f = 0.f;
        df = 0.f;
        return;
    }
    const float p = float(g.p);
    const float a = (p + 1.f) * (p + 2.f) * 0.5f, b = p * (p + 2.f), c = p * (p + 1.f) * 0.5f;
    const float xpm1 = powf(x, p - 1.f);
    const float xp = xpm1 * x;
    f = 1.f - a * xp + b * xp * x - c * xp * x * x;
    df = (-a * p * xpm1 + b * (p + 1.f) * xp - c * (p + 2.f) * xp * x) / g.r_max;
}

__global__ void edge_geometry_kernel(const float* __restrict__ pos, const float* __restrict__ cell,
                                     const int32_t* __restrict__ edge_index, const float* __restrict__ edge_image,
                                     int64_t n_edges, Geo g, float4* __restrict__ ysh, float* __restrict__ phi) {
    const float pref = sqrtf(2.0f / g.r_max);
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n_edges;
         e += int64_t(gridDim.x) * blockDim.x) {
        const float3 r = edge_vector(pos, cell, edge_index, edge_image, e);
        const float d = sqrtf((r.x * r.x + r.y * r.y) + r.z * r.z);
        float f, df;
        poly_cutoff(d, g, f, df);
        const bool ok = d > 0.f;
        const float inv = ok ? 1.0f / d : 0.f;
        ysh[e] = make_float4(kSqrt3 * r.x * inv, kSqrt3 * r.y * inv, kSqrt3 * r.z * inv, d);
        for (int n = 0; n < g.n_basis; ++n) {
            const float k = float(n + 1) * 3.14159265358979323846f / g.r_max;
            phi[e * g.n_basis + n] = ok ? pref * sinf(k * d) * inv * f : 0.f;
        }
    }
}

// d(loss)/d(r_e) of one edge from the gradients of its sqrt(3) u and phi
__device__ __forceinline__ float3 edge_grad_r(const float4 y, const float* gy, const float* gphi, const Geo& g) {
    const float d = y.w;
    if (!(d > 0.f)) return make_float3(0.f, 0.f, 0.f);
    const float inv = 1.0f / d;
    const float3 u = make_float3(y.x * kInvSqrt3, y.y * kInvSqrt3, y.z * kInvSqrt3);
    // Y1 = sqrt(3) r / d: dY_a/dr_b = sqrt(3) (delta_ab - u_a u_b) / d
    const float gu = (gy[0] * u.x + gy[1] * u.y) + gy[2] * u.z;
    float3 gr = make_float3(kSqrt3 * (gy[0] - gu * u.x) * inv, kSqrt3 * (gy[1] - gu * u.y) * inv,
                            kSqrt3 * (gy[2] - gu * u.z) * inv);
    float f, df;
    poly_cutoff(d, g, f, df);
    const float pref = sqrtf(2.0f / g.r_max);
    float gd = 0.f;
    for (int n = 0; n < g.n_basis; ++n) {
        const float k = float(n + 1) * 3.14159265358979323846f / g.r_max;
        float sn, cs;
        sincosf(k * d, &sn, &cs);
        const float b = pref * sn * inv;
        const float db = pref * (k * cs * d - sn) * inv * inv;
        gd += gphi[n] * (db * f + b * df);
    }
    gr.x += gd * u.x;
    gr.y += gd * u.y;
    gr.z += gd * u.z;
    return gr;
}

// Cell gradient and virial of the edge geometry: per edge g = d(loss)/d(r_e),
// image_grad[a][b] = sum_e image_e[a] g_b (d(loss)/d(cell), r_e = pos_j - pos_i
// + image_e . cell) and virial[a][b] = sum_e r_e[a] g_b. Deterministic: a fixed
// grid, each thread a fixed stride of edges summed in double, the CTA partials
// reduced in a fixed order by a second single-CTA pass.
constexpr int kVirialBlocks = 296, kVirialThreads = 256;
static_assert(FMD_EDGE_VIRIAL_WORKSPACE_DOUBLES >= kVirialBlocks * 18, "virial workspace");

__global__ void __launch_bounds__(kVirialThreads) edge_virial_partial_kernel(
    const float4* __restrict__ ysh, const float* __restrict__ gy, const float* __restrict__ gphi, Geo g,
    const float* __restrict__ edge_image, int64_t n_edges, const int64_t* __restrict__ n_real,
    double* __restrict__ partial) {
    __shared__ double red[kVirialThreads / 32][18];
    const int64_t n = n_real != nullptr ? min(*n_real, n_edges) : n_edges;
    double acc[18];
#pragma unroll
    for (int i = 0; i < 18; ++i) acc[i] = 0.0;
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
        const float4 y = ysh[e];
        const float3 gr = edge_grad_r(y, gy + 3 * e, gphi + e * g.n_basis, g);
        const float gv[3] = {gr.x, gr.y, gr.z};
        const float r[3] = {y.x * y.w * kInvSqrt3, y.y * y.w * kInvSqrt3, y.z * y.w * kInvSqrt3};
        const float im[3] = {edge_image[3 * e], edge_image[3 * e + 1], edge_image[3 * e + 2]};
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int b = 0; b < 3; ++b) {
                acc[3 * a + b] += double(im[a]) * double(gv[b]);
                acc[9 + 3 * a + b] += double(r[a]) * double(gv[b]);
            }
    }
#pragma unroll
    for (int i = 0; i < 18; ++i) {
        double v = acc[i];
        for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][i] = v;
    }
    __syncthreads();
    if (threadIdx.x < 18) {
        double v = 0.0;
        for (int w = 0; w < kVirialThreads / 32; ++w) v += red[w][threadIdx.x];
        partial[blockIdx.x * 18 + threadIdx.x] = v;
    }
}

__global__ void edge_virial_final_kernel(const double* __restrict__ partial, int blocks, float scale,
                                         float* __restrict__ image_grad, float* __restrict__ virial, int accumulate) {
    const int i = threadIdx.x;
    if (i >= 18) return;
    double v = 0.0;
    for (int b = 0; b < blocks; ++b) v += partial[b * 18 + i];
    float* out = i < 9 ? image_grad : virial;
    if (out == nullptr) return;
    const float x = float(v) * scale;
    out[i % 9] = accumulate ? out[i % 9] + x : x;
}

// dpos[a] = sum over edges sending from a of g_r - sum over edges received by a of g_r
__global__ void edge_geometry_bwd_kernel(const float4* __restrict__ ysh, const float* __restrict__ gy,
                                         const float* __restrict__ gphi, Geo g, const int32_t* __restrict__ edge_index,
                                         const int64_t* __restrict__ recv_off, const int64_t* __restrict__ send_off,
                                         const int32_t* __restrict__ send_perm, int64_t n_atoms,
                                         float* __restrict__ dpos, float scale, int accumulate) {
    for (int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; a < n_atoms;
         a += int64_t(gridDim.x) * blockDim.x) {
        float3 acc = make_float3(0.f, 0.f, 0.f);
        for (int64_t e = recv_off[a]; e < recv_off[a + 1]; ++e) {
            const float3 gr = edge_grad_r(ysh[e], gy + 3 * e, gphi + e * g.n_basis, g);
            acc.x -= gr.x;
            acc.y -= gr.y;
            acc.z -= gr.z;
        }
        for (int64_t t = send_off[a]; t < send_off[a + 1]; ++t) {
            const int64_t e = send_perm[t];
            const float3 gr = edge_grad_r(ysh[e], gy + 3 * e, gphi + e * g.n_basis, g);
            acc.x += gr.x;
            acc.y += gr.y;
            acc.z += gr.z;
        }
        acc = make_float3(scale * acc.x, scale * acc.y, scale * acc.z);
        if (accumulate) {
            dpos[3 * a] += acc.x;
            dpos[3 * a + 1] += acc.y;
            dpos[3 * a + 2] += acc.z;
        } else {
            dpos[3 * a] = acc.x;
            dpos[3 * a + 1] = acc.y;
            dpos[3 * a + 2] = acc.z;
        }
    }
}

// A_i = inv_avg * sum over the receiver run of the channel-wise tensor-product messages
template <int P>
__global__ void message_kernel(const float* __restrict__ R, const float* __restrict__ s_t,
                               const float* __restrict__ v_t, const float4* __restrict__ ysh,
                               const int32_t* __restrict__ edge_index, const int64_t* __restrict__ recv_off,
                               int64_t n_atoms, int C, float inv_avg, float* __restrict__ A0,
                               float* __restrict__ A1) {
    const int k = threadIdx.x;
    for (int64_t i = blockIdx.x; i < n_atoms; i += gridDim.x) {
        float a0 = 0.f, ax = 0.f, ay = 0.f, az = 0.f;
        for (int64_t e = recv_off[i]; e < recv_off[i + 1]; ++e) {
            const int64_t j = edge_index[2 * e + 1];
            const float4 y = ysh[e];
            const float* Re = R + e * (P * C);
            const float st = s_t[j * C + k];
            const float r0 = Re[k], r1 = Re[C + k];
            a0 += r0 * st;
            const float m1 = r1 * st;
            ax += m1 * y.x;
            ay += m1 * y.y;
            az += m1 * y.z;
            if constexpr (P == 4) {
                const float vx = v_t[j * 3 * C + k], vy = v_t[j * 3 * C + C + k], vz = v_t[j * 3 * C + 2 * C + k];
                const float r2 = Re[2 * C + k], r3 = Re[3 * C + k];
                ax += r2 * vx;
                ay += r2 * vy;
                az += r2 * vz;
                a0 += r3 * ((vx * y.x + vy * y.y) + vz * y.z) * kInvSqrt3;
            }
        }
        A0[i * C + k] = a0 * inv_avg;
        A1[i * 3 * C + k] = ax * inv_avg;
        A1[i * 3 * C + C + k] = ay * inv_avg;
        A1[i * 3 * C + 2 * C + k] = az * inv_avg;
    }
}

// per-edge gradients: dR [E, P*C] and dY [E, 3] (block reduction over channels)
template <int P>
__global__ void message_bwd_edge_kernel(const float* __restrict__ dA0, const float* __restrict__ dA1,
                                        const float* __restrict__ R, const float* __restrict__ s_t,
                                        const float* __restrict__ v_t, const float4* __restrict__ ysh,
                                        const int32_t* __restrict__ edge_index, const int64_t* __restrict__ recv_off,
                                        int64_t n_atoms, int C, float inv_avg, float* __restrict__ dR,
                                        float* __restrict__ dY, int accumulate_dy) {
    __shared__ float s_part[32][3];
    const int k = threadIdx.x, lane = k & 31, warp = k >> 5, nwarps = blockDim.x >> 5;
    for (int64_t i = blockIdx.x; i < n_atoms; i += gridDim.x) {
        const float g0 = dA0[i * C + k] * inv_avg;
        const float gx = dA1[i * 3 * C + k] * inv_avg, gy_ = dA1[i * 3 * C + C + k] * inv_avg,
                    gz = dA1[i * 3 * C + 2 * C + k] * inv_avg;
        for (int64_t e = recv_off[i]; e < recv_off[i + 1]; ++e) {
            const int64_t j = edge_index[2 * e + 1];
            const float4 y = ysh[e];
            const float* Re = R + e * (P * C);
            float* dRe = dR + e * (P * C);
            const float st = s_t[j * C + k];
            const float gdoty = (gx * y.x + gy_ * y.y) + gz * y.z;
            dRe[k] = g0 * st;
            dRe[C + k] = st * gdoty;
            const float c1 = Re[C + k] * st;
            float px = c1 * gx, py = c1 * gy_, pz = c1 * gz;
            if constexpr (P == 4) {
                const float vx = v_t[j * 3 * C + k], vy = v_t[j * 3 * C + C + k], vz = v_t[j * 3 * C + 2 * C + k];
                dRe[2 * C + k] = (gx * vx + gy_ * vy) + gz * vz;
                dRe[3 * C + k] = g0 * ((vx * y.x + vy * y.y) + vz * y.z) * kInvSqrt3;
                const float c3 = Re[3 * C + k] * g0 * kInvSqrt3;
                px += c3 * vx;
                py += c3 * vy;
                pz += c3 * vz;
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) {
                px += __shfl_xor_sync(0xffffffffu, px, m);
                py += __shfl_xor_sync(0xffffffffu, py, m);
                pz += __shfl_xor_sync(0xffffffffu, pz, m);
            }
            if (lane == 0) {
                s_part[warp][0] = px;
                s_part[warp][1] = py;
                s_part[warp][2] = pz;
            }
            __syncthreads();
            if (k < 3) {
                float t = 0.f;
                for (int w = 0; w < nwarps; ++w) t += s_part[w][k];
                dY[3 * e + k] = accumulate_dy ? dY[3 * e + k] + t : t;
            }
            __syncthreads();
        }
    }
}

// per-sender gradients of the gathered rows: ds_t [N, C], dv_t [N, 3, C]
template <int P>
__global__ void message_bwd_sender_kernel(const float* __restrict__ dA0, const float* __restrict__ dA1,
                                          const float* __restrict__ R, const float4* __restrict__ ysh,
                                          const int32_t* __restrict__ edge_index, const int64_t* __restrict__ send_off,
                                          const int32_t* __restrict__ send_perm, int64_t n_atoms, int C,
                                          float inv_avg, float* __restrict__ ds, float* __restrict__ dv) {
    const int k = threadIdx.x;
    for (int64_t j = blockIdx.x; j < n_atoms; j += gridDim.x) {
        float s_acc = 0.f, vx = 0.f, vy = 0.f, vz = 0.f;
        for (int64_t t = send_off[j]; t < send_off[j + 1]; ++t) {
            const int64_t e = send_perm[t];
            const int64_t i = edge_index[2 * e];
            const float4 y = ysh[e];
            const float* Re = R + e * (P * C);
            const float g0 = dA0[i * C + k] * inv_avg;
            const float gx = dA1[i * 3 * C + k] * inv_avg, gy_ = dA1[i * 3 * C + C + k] * inv_avg,
                        gz = dA1[i * 3 * C + 2 * C + k] * inv_avg;
            s_acc += Re[k] * g0 + Re[C + k] * ((gx * y.x + gy_ * y.y) + gz * y.z);
            if constexpr (P == 4) {
                const float r2 = Re[2 * C + k];
                const float r3 = Re[3 * C + k] * g0 * kInvSqrt3;
                vx += r2 * gx + r3 * y.x;
                vy += r2 * gy_ + r3 * y.y;
                vz += r2 * gz + r3 * y.z;
            }
        }
        ds[j * C + k] = s_acc;
        if constexpr (P == 4) {
            dv[j * 3 * C + k] = vx;
            dv[j * 3 * C + C + k] = vy;
            dv[j * 3 * C + 2 * C + k] = vz;
        }
    }
}

// symmetric contraction of correlation 3 for l <= 1, per (atom, channel), element weights:
//   B0 = w0 a + w1 a^2 + w2 q + w3 a^3 + w4 a q            (q = V.V)
//   B1 = (u0 + u1 a + u2 a^2 + u3 q) V
__global__ void product_kernel(const float* __restrict__ A0, const float* __restrict__ A1,
                               const int32_t* __restrict__ elem, const float* __restrict__ W0,
                               const float* __restrict__ W1, int64_t n_atoms, int C, float* __restrict__ B0,
                               float* __restrict__ B1) {
    const int64_t total = n_atoms * C;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = t / C;
        const int k = int(t - i * C);
        const int64_t z = elem[i];
        const float a = A0[t];
        const float vx = A1[i * 3 * C + k], vy = A1[i * 3 * C + C + k], vz = A1[i * 3 * C + 2 * C + k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float* w = W0 + z * 5 * C + k;
        B0[t] = (((w[0] * a + w[C] * a * a) + w[2 * C] * q) + w[3 * C] * a * a * a) + w[4 * C] * a * q;
        if (B1 != nullptr) {
            const float* u = W1 + z * 4 * C + k;
            const float c = ((u[0] + u[C] * a) + u[2 * C] * a * a) + u[3 * C] * q;
            B1[i * 3 * C + k] = c * vx;
            B1[i * 3 * C + C + k] = c * vy;
            B1[i * 3 * C + 2 * C + k] = c * vz;
        }
    }
}

__global__ void product_bwd_kernel(const float* __restrict__ dB0, const float* __restrict__ dB1,
                                   const float* __restrict__ A0, const float* __restrict__ A1,
                                   const int32_t* __restrict__ elem, const float* __restrict__ W0,
                                   const float* __restrict__ W1, int64_t n_atoms, int C, float* __restrict__ dA0,
                                   float* __restrict__ dA1) {
    const int64_t total = n_atoms * C;
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = t / C;
        const int k = int(t - i * C);
        const int64_t z = elem[i];
        const float a = A0[t];
        const float vx = A1[i * 3 * C + k], vy = A1[i * 3 * C + C + k], vz = A1[i * 3 * C + 2 * C + k];
        const float q = (vx * vx + vy * vy) + vz * vz;
        const float* w = W0 + z * 5 * C + k;
        const float g0 = dB0[t];
        float ga = g0 * (((w[0] + 2.f * w[C] * a) + 3.f * w[3 * C] * a * a) + w[4 * C] * q);
        float gq = g0 * (w[2 * C] + w[4 * C] * a);
        float gx = 0.f, gy = 0.f, gz = 0.f;
        if (dB1 != nullptr) {
            const float* u = W1 + z * 4 * C + k;
            const float c = ((u[0] + u[C] * a) + u[2 * C] * a * a) + u[3 * C] * q;
            const float bx = dB1[i * 3 * C + k], by = dB1[i * 3 * C + C + k], bz = dB1[i * 3 * C + 2 * C + k];
            const float bv = (bx * vx + by * vy) + bz * vz;
            ga += bv * (u[C] + 2.f * u[2 * C] * a);
            gq += bv * u[3 * C];
            gx = c * bx;
            gy = c * by;
            gz = c * bz;
        }
        dA0[t] = ga;
        dA1[i * 3 * C + k] = gx + 2.f * gq * vx;
        dA1[i * 3 * C + C + k] = gy + 2.f * gq * vy;
        dA1[i * 3 * C + 2 * C + k] = gz + 2.f * gq * vz;
    }
}

// y[r, :] (+)= x[r, :] @ W[z(r)]   (W[z] [C_in, C_out]; transposed: x @ W[z]^T, W[z] [C_out, C_in])
// z(r) = elem[r / rows_per_atom]; one CTA per row, one thread per output column
__global__ void element_linear_kernel(const float* __restrict__ x, int64_t rows, int rows_per_atom,
                                      const int32_t* __restrict__ elem, const float* __restrict__ W, int c_in,
                                      int c_out, int transpose, float* __restrict__ y, int accumulate) {
    extern __shared__ float s_x[];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        __syncthreads();
        for (int c = threadIdx.x; c < c_in; c += blockDim.x) s_x[c] = x[r * c_in + c];
        __syncthreads();
        const int64_t z = elem[r / rows_per_atom];
        const float* Wz = W + z * int64_t(c_in) * c_out;
        for (int o = threadIdx.x; o < c_out; o += blockDim.x) {
            float acc = 0.f;
            if (transpose) {
                for (int c = 0; c < c_in; ++c) acc = fmaf(s_x[c], Wz[int64_t(o) * c_in + c], acc);
            } else {
                for (int c = 0; c < c_in; ++c) acc = fmaf(s_x[c], Wz[int64_t(c) * c_out + o], acc);
            }
            float* dst = y + r * c_out + o;
            *dst = accumulate ? *dst + acc : acc;
        }
    }
}

// per-atom energy E_i = E0[z_i] + scale * (sum_t e_t[i]) + shift (fp64) and per-system sums
__global__ void node_energy_kernel(const float* __restrict__ e_terms, int n_terms, int64_t ld_terms,
                                   const int32_t* __restrict__ elem, const double* __restrict__ e0,
                                   double scale, double shift, int64_t n_atoms, double* __restrict__ node_energy,
                                   double* __restrict__ total) {
    __shared__ double s_part[32];
    const int64_t sys = blockIdx.x;
    double acc = 0.0;
    for (int64_t a = threadIdx.x; a < n_atoms; a += blockDim.x) {
        const int64_t i = sys * n_atoms + a;
        double t = 0.0;
        for (int k = 0; k < n_terms; ++k) t += double(e_terms[k * ld_terms + i]);
        const double ei = e0[elem[i]] + scale * t + shift;
        node_energy[i] = ei;
        acc += ei;
    }
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += s_part[w];
        total[sys] = s;
    }
}

// gradient of the per-system totals with respect to every energy term of every atom
__global__ void node_energy_bwd_kernel(const double* __restrict__ d_total, double scale, int64_t n_atoms,
                                       int32_t n_systems, float* __restrict__ d_term) {
    const int64_t total = n_atoms * n_systems;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
         i += int64_t(gridDim.x) * blockDim.x)
        d_term[i] = float(scale * d_total[i / n_atoms]);
}

inline bool geo_ok(const Geo& g) { return g.r_max > 0.f && g.n_basis >= 1 && g.n_basis <= kMaxBasis && g.p >= 1; }

}  // namespace fmd

using namespace fmd;

extern "C" {

fmd_status fmd_mace_edge_geometry(const float* positions, const float* cell, const int32_t* edge_index,
                                  const float* edge_image, int64_t n_edges, float r_max, int32_t n_basis,
                                  int32_t poly_p, float* ysh, float* phi, void* stream) {
    const Geo g{r_max, n_basis, poly_p};
    if (positions == nullptr || cell == nullptr || edge_index == nullptr || edge_image == nullptr ||
        ysh == nullptr || phi == nullptr || n_edges < 0 || !geo_ok(g) || !aligned16(ysh))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_edges == 0) return FMD_OK;
    edge_geometry_kernel<<<grid_for(n_edges, 256), 256, 0, as_stream(stream)>>>(
        positions, cell, edge_index, edge_image, n_edges, g, reinterpret_cast<float4*>(ysh), phi);
    return check_launch();
}

fmd_status fmd_mace_edge_geometry_bwd(const float* ysh, const float* grad_y, const float* grad_phi, float r_max,
                                      int32_t n_basis, int32_t poly_p, const int32_t* edge_index,
                                      const int64_t* recv_off, const int64_t* send_off, const int32_t* send_perm,
                                      int64_t n_atoms, float* grad_positions, float scale, int32_t accumulate,
                                      void* stream) {
    const Geo g{r_max, n_basis, poly_p};
    if (ysh == nullptr || grad_y == nullptr || grad_phi == nullptr || edge_index == nullptr ||
        recv_off == nullptr || send_off == nullptr || send_perm == nullptr || grad_positions == nullptr ||
        n_atoms < 0 || !geo_ok(g) || !aligned16(ysh))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    edge_geometry_bwd_kernel<<<grid_for(n_atoms, 128), 128, 0, as_stream(stream)>>>(
        reinterpret_cast<const float4*>(ysh), grad_y, grad_phi, g, edge_index, recv_off, send_off, send_perm,
        n_atoms, grad_positions, scale, accumulate);
    return check_launch();
}

fmd_status fmd_mace_edge_virial(const float* ysh, const float* grad_y, const float* grad_phi, float r_max,
                                int32_t n_basis, int32_t poly_p, const float* edge_image, int64_t n_edges,
                                const int64_t* n_real_edges, double* workspace, float scale, float* image_grad,
                                float* virial, int32_t accumulate, void* stream) {
    const Geo g{r_max, n_basis, poly_p};
    if (ysh == nullptr || grad_y == nullptr || grad_phi == nullptr || edge_image == nullptr || workspace == nullptr ||
        n_edges < 0 || !geo_ok(g) || !aligned16(ysh) || (image_grad == nullptr && virial == nullptr))
        return FMD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = as_stream(stream);
    edge_virial_partial_kernel<<<kVirialBlocks, kVirialThreads, 0, st>>>(
        reinterpret_cast<const float4*>(ysh), grad_y, grad_phi, g, edge_image, n_edges, n_real_edges, workspace);
    edge_virial_final_kernel<<<1, 32, 0, st>>>(workspace, kVirialBlocks, scale, image_grad, virial, accumulate);
    return check_launch();
}

static bool channels_ok(int32_t C) { return C >= 32 && C <= 1024 && C % 32 == 0; }

fmd_status fmd_mace_message(const float* R, int32_t n_paths, const float* s_t, const float* v_t,
                            const float* ysh, const int32_t* edge_index, const int64_t* recv_off,
                            int64_t n_atoms, int32_t channels, float inv_avg, float* A0, float* A1,
                            void* stream) {
    if (R == nullptr || s_t == nullptr || ysh == nullptr || edge_index == nullptr || recv_off == nullptr ||
        A0 == nullptr || A1 == nullptr || n_atoms < 0 || !channels_ok(channels) ||
        (n_paths != 2 && n_paths != 4) || (n_paths == 4 && v_t == nullptr) || !aligned16(ysh))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    const int grid = int(n_atoms < int64_t(kNumSMs) * 32 ? n_atoms : int64_t(kNumSMs) * 32);
    const float4* y = reinterpret_cast<const float4*>(ysh);
    if (n_paths == 2)
        message_kernel<2><<<grid, channels, 0, as_stream(stream)>>>(R, s_t, v_t, y, edge_index, recv_off, n_atoms,
                                                                    channels, inv_avg, A0, A1);
    else
        message_kernel<4><<<grid, channels, 0, as_stream(stream)>>>(R, s_t, v_t, y, edge_index, recv_off, n_atoms,
                                                                    channels, inv_avg, A0, A1);
    return check_launch();
}

fmd_status fmd_mace_message_bwd(const float* dA0, const float* dA1, const float* R, int32_t n_paths,
                                const float* s_t, const float* v_t, const float* ysh, const int32_t* edge_index,
                                const int64_t* recv_off, const int64_t* send_off, const int32_t* send_perm,
                                int64_t n_atoms, int32_t channels, float inv_avg, float* dR, float* dY,
                                int32_t accumulate_dy, float* ds_t, float* dv_t, void* stream) {
    if (dA0 == nullptr || dA1 == nullptr || R == nullptr || s_t == nullptr || ysh == nullptr ||
        edge_index == nullptr || recv_off == nullptr || send_off == nullptr || send_perm == nullptr ||
        dR == nullptr || dY == nullptr || ds_t == nullptr || n_atoms < 0 || !channels_ok(channels) ||
        (n_paths != 2 && n_paths != 4) || (n_paths == 4 && (v_t == nullptr || dv_t == nullptr)) ||
        !aligned16(ysh))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    const int grid = int(n_atoms < int64_t(kNumSMs) * 32 ? n_atoms : int64_t(kNumSMs) * 32);
    const float4* y = reinterpret_cast<const float4*>(ysh);
    cudaStream_t s = as_stream(stream);
    if (n_paths == 2) {
        message_bwd_edge_kernel<2><<<grid, channels, 0, s>>>(dA0, dA1, R, s_t, v_t, y, edge_index, recv_off, n_atoms,
                                                             channels, inv_avg, dR, dY, accumulate_dy);
        message_bwd_sender_kernel<2><<<grid, channels, 0, s>>>(dA0, dA1, R, y, edge_index, send_off, send_perm,
                                                               n_atoms, channels, inv_avg, ds_t, dv_t);
    } else {
        message_bwd_edge_kernel<4><<<grid, channels, 0, s>>>(dA0, dA1, R, s_t, v_t, y, edge_index, recv_off, n_atoms,
                                                             channels, inv_avg, dR, dY, accumulate_dy);
        message_bwd_sender_kernel<4><<<grid, channels, 0, s>>>(dA0, dA1, R, y, edge_index, send_off, send_perm,
                                                               n_atoms, channels, inv_avg, ds_t, dv_t);
    }
    return check_launch();
}

fmd_status fmd_mace_product(const float* A0, const float* A1, const int32_t* elem, const float* W0,
                            const float* W1, int64_t n_atoms, int32_t channels, float* B0, float* B1,
                            void* stream) {
    if (A0 == nullptr || A1 == nullptr || elem == nullptr || W0 == nullptr || B0 == nullptr || n_atoms < 0 ||
        channels < 1 || ((W1 == nullptr) != (B1 == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    product_kernel<<<grid_for(n_atoms * channels, 256), 256, 0, as_stream(stream)>>>(A0, A1, elem, W0, W1, n_atoms,
                                                                                    channels, B0, B1);
    return check_launch();
}

fmd_status fmd_mace_product_bwd(const float* dB0, const float* dB1, const float* A0, const float* A1,
                                const int32_t* elem, const float* W0, const float* W1, int64_t n_atoms,
                                int32_t channels, float* dA0, float* dA1, void* stream) {
    if (dB0 == nullptr || A0 == nullptr || A1 == nullptr || elem == nullptr || W0 == nullptr || dA0 == nullptr ||
        dA1 == nullptr || n_atoms < 0 || channels < 1 || ((W1 == nullptr) != (dB1 == nullptr)))
        return FMD_ERR_INVALID_ARGUMENT;
    if (n_atoms == 0) return FMD_OK;
    product_bwd_kernel<<<grid_for(n_atoms * channels, 256), 256, 0, as_stream(stream)>>>(
        dB0, dB1, A0, A1, elem, W0, W1, n_atoms, channels, dA0, dA1);
    return check_launch();
}

fmd_status fmd_element_linear(const float* x, int64_t rows, int32_t rows_per_atom, const int32_t* elem,
                              const float* W, int32_t c_in, int32_t c_out, int32_t transpose, float* y,
                              int32_t accumulate, void* stream) {
    if (x == nullptr || elem == nullptr || W == nullptr || y == nullptr || rows < 0 || rows_per_atom < 1 ||
        c_in < 1 || c_out < 1 || c_in > 8192)
        return FMD_ERR_INVALID_ARGUMENT;
    if (rows == 0) return FMD_OK;
    const int threads = c_out >= 128 ? 128 : 32 * ((c_out + 31) / 32);
    const int grid = int(rows < int64_t(kNumSMs) * 32 ? rows : int64_t(kNumSMs) * 32);
    element_linear_kernel<<<grid, threads, sizeof(float) * c_in, as_stream(stream)>>>(
        x, rows, rows_per_atom, elem, W, c_in, c_out, transpose, y, accumulate);
    return check_launch();
}

fmd_status fmd_mace_node_energy(const float* e_terms, int32_t n_terms, int64_t ld_terms, const int32_t* elem,
                                const double* e0, double scale, double shift, int64_t n_atoms, int32_t n_systems,
                                double* node_energy, double* total, void* stream) {
    if (e_terms == nullptr || elem == nullptr || e0 == nullptr || node_energy == nullptr || total == nullptr ||
        n_terms < 1 || n_atoms < 1 || n_systems < 1 || ld_terms < n_atoms * n_systems)
        return FMD_ERR_INVALID_ARGUMENT;
    node_energy_kernel<<<n_systems, 256, 0, as_stream(stream)>>>(e_terms, n_terms, ld_terms, elem, e0, scale, shift,
                                                                 n_atoms, node_energy, total);
    return check_launch();
}

fmd_status fmd_mace_node_energy_bwd(const double* d_total, double scale, int64_t n_atoms, int32_t n_systems,
                                    float* d_term, void* stream) {
    if (d_total == nullptr || d_term == nullptr || n_atoms < 1 || n_systems < 1) return FMD_ERR_INVALID_ARGUMENT;
    node_energy_bwd_kernel<<<grid_for(n_atoms * n_systems, 256), 256, 0, as_stream(stream)>>>(d_total, scale, n_atoms,
                                                                                           n_systems, d_term);
    return check_launch();
}

}  // extern "C"
